// tokens.cpp -- IPA text -> Kokoro token ids and the chunking of long IPA
// text (rokoko::to_tokens / chunk_ipa, src/rokoko.h:141-221), the data format
// between the phonemizer's output and the model's input.  Host code only.
#include <algorithm>
#include <cstddef>
#include <cstdint>

#include "../../include/rk_b200.h"
#include "status.h"

namespace rk {

namespace {

// The model's input vocabulary: IPA / punctuation code point -> token id
// (the embedding row), sorted by code point.  Anything else is dropped.
struct Sym {
    uint32_t cp;
    int32_t id;
};
constexpr Sym kVocab[] = {
    {0x0020, 16}, {0x0021, 5}, {0x0022, 11}, {0x0028, 12}, {0x0029, 13}, {0x002C, 3},
    {0x002E, 4}, {0x003A, 2}, {0x003B, 1}, {0x003F, 6}, {0x0041, 24}, {0x0049, 25},
    {0x004F, 31}, {0x0051, 33}, {0x0053, 35}, {0x0054, 36}, {0x0057, 39}, {0x0059, 41},
    {0x0061, 43}, {0x0062, 44}, {0x0063, 45}, {0x0064, 46}, {0x0065, 47}, {0x0066, 48},
    {0x0068, 50}, {0x0069, 51}, {0x006A, 52}, {0x006B, 53}, {0x006C, 54}, {0x006D, 55},
    {0x006E, 56}, {0x006F, 57}, {0x0070, 58}, {0x0071, 59}, {0x0072, 60}, {0x0073, 61},
    {0x0074, 62}, {0x0075, 63}, {0x0076, 64}, {0x0077, 65}, {0x0078, 66}, {0x0079, 67},
    {0x007A, 68}, {0x00E6, 72}, {0x00E7, 78}, {0x00F0, 81}, {0x00F8, 116}, {0x014B, 112},
    {0x0153, 120}, {0x0250, 70}, {0x0251, 69}, {0x0252, 71}, {0x0254, 76}, {0x0255, 77},
    {0x0256, 80}, {0x0259, 83}, {0x025A, 85}, {0x025B, 86}, {0x025C, 87}, {0x025F, 90},
    {0x0261, 92}, {0x0263, 139}, {0x0264, 140}, {0x0265, 99}, {0x0268, 101}, {0x026A, 102},
    {0x026F, 110}, {0x0270, 111}, {0x0272, 114}, {0x0273, 113}, {0x0274, 115}, {0x0278, 118},
    {0x0279, 123}, {0x027B, 126}, {0x027D, 129}, {0x027E, 125}, {0x0281, 128}, {0x0282, 130},
    {0x0283, 131}, {0x0288, 132}, {0x028A, 135}, {0x028B, 136}, {0x028C, 138}, {0x028E, 143},
    {0x0292, 147}, {0x0294, 148}, {0x029D, 103}, {0x02A3, 18}, {0x02A4, 82}, {0x02A5, 19},
    {0x02A6, 20}, {0x02A7, 133}, {0x02A8, 21}, {0x02B0, 162}, {0x02B2, 164}, {0x02C8, 156},
    {0x02CC, 157}, {0x02D0, 158}, {0x0303, 17}, {0x03B2, 75}, {0x03B8, 119}, {0x03C7, 142},
    {0x1D4A, 42}, {0x1D5D, 22}, {0x1D7B, 177}, {0x2014, 9}, {0x201C, 14}, {0x201D, 15},
    {0x2026, 10}, {0x2192, 171}, {0x2193, 169}, {0x2197, 172}, {0x2198, 173}, {0xAB67, 23},
};

int32_t token_of(uint32_t cp) {
    const Sym* end = kVocab + sizeof(kVocab) / sizeof(kVocab[0]);
    const Sym* it = std::lower_bound(kVocab, end, cp, [](const Sym& s, uint32_t v) { return s.cp < v; });
    return (it != end && it->cp == cp) ? it->id : -1;
}

// one code point starting at s[i]: the lead byte gives the length, continuation
// bytes are taken as they come (the reference's decoder), i advances past it
uint32_t next_cp(const unsigned char* s, size_t n, size_t& i) {
    const unsigned char c = s[i];
    if (c < 0x80) { i++; return c; }
    uint32_t cp;
    int extra;
    if ((c & 0xE0) == 0xC0) { cp = c & 0x1F; extra = 1; }
    else if ((c & 0xF0) == 0xE0) { cp = c & 0x0F; extra = 2; }
    else { cp = c & 0x07; extra = 3; }
    i++;
    for (int j = 0; j < extra && i < n; j++, i++) cp = (cp << 6) | (s[i] & 0x3F);
    return cp;
}

size_t count_cps(const unsigned char* s, size_t n) {
    size_t i = 0, k = 0;
    while (i < n) { next_cp(s, n, i); k++; }
    return k;
}

// byte offset after the first `cps` code points
size_t offset_of(const unsigned char* s, size_t n, size_t cps) {
    size_t i = 0, k = 0;
    while (i < n && k < cps) { next_cp(s, n, i); k++; }
    return i;
}

constexpr size_t kMaxChunk = 510;  // code points per chunk (src/rokoko.h:159)

// last position j in (0, limit] with s[j - 1] in `set`, or 0
size_t last_of(const unsigned char* s, size_t limit, const char* set) {
    for (size_t j = limit; j > 0; j--)
        for (const char* c = set; *c; c++)
            if (s[j - 1] == (unsigned char)*c) return j;
    return 0;
}

}  // namespace

}  // namespace rk

using namespace rk;

extern "C" rk_status rk_ipa_to_tokens(const char* ipa, size_t bytes, int32_t* ids, size_t cap, size_t* count) {
    if ((!ipa && bytes) || !count) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_ipa_to_tokens: bad arguments");
    const unsigned char* s = reinterpret_cast<const unsigned char*>(ipa);
    size_t k = 0;
    auto put = [&](int32_t v) {
        if (ids && k < cap) ids[k] = v;
        k++;
    };
    put(0);  // BOS
    size_t i = 0;
    while (i < bytes) {
        const int32_t t = token_of(next_cp(s, bytes, i));
        if (t >= 0) put(t);
    }
    put(0);  // EOS
    *count = k;
    if (ids && k > cap) return fail(RK_ERR_WORKSPACE, "rk_ipa_to_tokens: ids buffer too small (*count = needed)");
    return RK_OK;
}

extern "C" rk_status rk_ipa_chunks(const char* ipa, size_t bytes, size_t* ends, size_t cap, size_t* n) {
    if ((!ipa && bytes) || !n) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_ipa_chunks: bad arguments");
    const unsigned char* s = reinterpret_cast<const unsigned char*>(ipa);
    size_t k = 0;
    auto put = [&](size_t e) {
        if (ends && k < cap) ends[k] = e;
        k++;
    };
    if (count_cps(s, bytes) <= kMaxChunk) {
        put(bytes);
    } else {
        size_t pos = 0;
        while (pos < bytes) {
            const unsigned char* rest = s + pos;
            const size_t left = bytes - pos;
            if (count_cps(rest, left) <= kMaxChunk) { put(bytes); break; }
            // split after the last sentence mark within 510 code points, else the last
            // clause mark, else the last space, else at the limit
            const size_t limit = offset_of(rest, left, kMaxChunk);
            size_t split = last_of(rest, limit, ".!?");
            if (!split) split = last_of(rest, limit, ",:;");
            if (!split) split = last_of(rest, limit, " ");
            if (!split) split = limit;
            pos += split;
            put(pos);
        }
    }
    *n = k;
    if (ends && k > cap) return fail(RK_ERR_WORKSPACE, "rk_ipa_chunks: ends buffer too small (*n = needed)");
    return RK_OK;
}
