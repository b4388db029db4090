// oracle/g2p.cpp -- CPU FP32 restatement of rokoko's neural phonemizer
// (G2P3 Conformer-CTC, src/g2p.h).
//
// TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); never part
// of the product path.
//
// Steps, each after the reference's own (file:line of src/g2p.h):
//   UTF-8 -> code points -> char ids (unknown -> 0)              :682-694
//   X = char_emb[id]                                             :326-335 (g2p_embed_kernel)
//   per layer:
//     h = RMSNorm(X; n1_w, eps 1e-6)                             :55-80, :755-757
//     QKV = h Wqkv^T + bqkv; RoPE on Q and K (per head, halves)  :759-770, :171-205
//       cos/sin tables: freq = t / 10000^(2i/head_dim) in float  :558-568
//     S = Q K^T / sqrt(head_dim) per head, softmax over keys     :772-790, :105-142
//     A = P V; X += A Wout^T + bout                              :784-799
//     h = RMSNorm(X; n2_w); G = h Wgate^T + bg, U = h Wup^T + bu :797-807
//     X += (G sigmoid(G) U) Wdown^T + bdown                      :807-815, :144-156
//   P = X Wup^T + bup, row t -> rows t*up .. t*up+up-1           :817-823, :337-351
//   logits = P Wh^T + bh; argmax per row (first maximum)         :825-832, :353-366
//   CTC: drop blank 0 and repeats, id -> phone code point -> UTF-8   :865-882
//   inputs longer than max_pos_ = 2048 characters give ""       :416, :697
// Products and sums are FP32; the GEMMs use the oracle's blocked kernel
// (gemm.cpp), whose summation order differs from the reference's TF32
// tensor-core GEMMs, so logits agree to a tolerance, not bitwise.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "oracle_internal.h"

namespace {

struct Layer {
    std::vector<float> n1, wqkv_t, bqkv, wout_t, bout, n2, wgate_t, bgate, wup_t, bup, wdown_t, bdown;
};

struct G2P {
    int d = 0, heads = 0, n_layers = 0, ff = 0, up = 0, n_chars = 0, n_phones = 0, dk = 0;
    static constexpr int kMaxPos = 2048;
    std::unordered_map<uint32_t, int> char2id;
    std::unordered_map<int, uint32_t> id2phone;
    std::vector<float> emb, rope_cos, rope_sin;
    std::vector<Layer> layers;
    std::vector<float> wupp_t, bupp, whead_t, bhead;
};

// [out][in] -> [in][out] (the oracle's GEMM reads B row-major [K][N])
std::vector<float> transpose(const float* w, int out, int in) {
    std::vector<float> t((size_t)out * in);
    for (int o = 0; o < out; o++)
        for (int i = 0; i < in; i++) t[(size_t)i * out + o] = w[(size_t)o * in + i];
    return t;
}

// y[T][out] = x[T][in] W^T (+ bias)
void linear(const float* x, int T, int in, const std::vector<float>& w_t, const std::vector<float>& b, int out,
            float* y) {
    for (int t = 0; t < T; t++)
        for (int o = 0; o < out; o++) y[(size_t)t * out + o] = 0.f;
    orc::gemm_acc(T, out, in, x, in, w_t.data(), out, y, out);
    if (!b.empty())
        for (int t = 0; t < T; t++)
            for (int o = 0; o < out; o++) y[(size_t)t * out + o] += b[o];
}

void rms_norm(const float* x, const std::vector<float>& w, int T, int d, float* out) {
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * d;
        float ss = 0.f;
        for (int i = 0; i < d; i++) ss += xt[i] * xt[i];
        const float inv = 1.0f / std::sqrt(ss / d + 1e-6f);
        for (int i = 0; i < d; i++) out[(size_t)t * d + i] = w[i] * xt[i] * inv;
    }
}

std::vector<uint32_t> codepoints(const char* s, size_t n) {
    // the reference's lenient decoder: lead byte decides the length, continuation bits taken as they come
    std::vector<uint32_t> cps;
    const uint8_t* p = (const uint8_t*)s;
    const uint8_t* end = p + n;
    while (p < end) {
        uint32_t cp;
        if (*p < 0x80) {
            cp = *p++;
        } else if ((*p & 0xE0) == 0xC0) {
            cp = (*p++ & 0x1Fu) << 6;
            if (p < end) cp |= (*p++ & 0x3Fu);
        } else if ((*p & 0xF0) == 0xE0) {
            cp = (*p++ & 0x0Fu) << 12;
            if (p < end) cp |= (*p++ & 0x3Fu) << 6;
            if (p < end) cp |= (*p++ & 0x3Fu);
        } else {
            cp = (*p++ & 0x07u) << 18;
            if (p < end) cp |= (*p++ & 0x3Fu) << 12;
            if (p < end) cp |= (*p++ & 0x3Fu) << 6;
            if (p < end) cp |= (*p++ & 0x3Fu);
        }
        cps.push_back(cp);
    }
    return cps;
}

void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xF0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3F));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

struct Reader {
    const uint8_t* p;
    size_t n, off = 0;
    bool u32(uint32_t& v) {
        if (off + 4 > n) return false;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return true;
    }
    bool f32(std::vector<float>& v, size_t cnt) {
        if (off + 4 * cnt > n) return false;
        v.resize(cnt);
        std::memcpy(v.data(), p + off, 4 * cnt);
        off += 4 * cnt;
        return true;
    }
};

// X [T][d] -> logits [T*up][n_phones]
void forward(const G2P& m, const std::vector<int>& ids, std::vector<float>& logits) {
    const int T = (int)ids.size(), d = m.d, dk = m.dk, d2 = dk / 2, ff = m.ff, H = m.heads;
    std::vector<float> X((size_t)T * d), h((size_t)T * d), qkv((size_t)T * 3 * d), att((size_t)T * d),
        tmp((size_t)T * d), gu((size_t)T * ff), uu((size_t)T * ff);
    for (int t = 0; t < T; t++) std::memcpy(&X[(size_t)t * d], &m.emb[(size_t)ids[t] * d], d * 4);
    const float scale = 1.0f / std::sqrt((float)dk);
    for (const Layer& L : m.layers) {
        rms_norm(X.data(), L.n1, T, d, h.data());
        linear(h.data(), T, d, L.wqkv_t, L.bqkv, 3 * d, qkv.data());
        for (int t = 0; t < T; t++)
            for (int hh = 0; hh < H; hh++)
                for (int part = 0; part < 2; part++) {  // Q, then K
                    float* b = &qkv[(size_t)t * 3 * d + part * d + hh * dk];
                    for (int i = 0; i < d2; i++) {
                        const float c = m.rope_cos[(size_t)t * d2 + i], s = m.rope_sin[(size_t)t * d2 + i];
                        const float x0 = b[i], x1 = b[d2 + i];
                        b[i] = x0 * c - x1 * s;
                        b[d2 + i] = x1 * c + x0 * s;
                    }
                }
        // work items = (head, block of 64 queries); each query's arithmetic is the same in any split
        const int qblk = (T + 63) / 64;
        orc::parallel_for(H * qblk, [&](int item) {
            const int hh = item / qblk, q0 = (item % qblk) * 64, q1 = std::min(T, q0 + 64);
            std::vector<float> p(T);
            for (int q = q0; q < q1; q++) {
                const float* qv = &qkv[(size_t)q * 3 * d + hh * dk];
                float mx = -1e30f;
                for (int k = 0; k < T; k++) {
                    const float* kv = &qkv[(size_t)k * 3 * d + d + hh * dk];
                    float s = 0.f;
                    for (int i = 0; i < dk; i++) s += qv[i] * kv[i];
                    p[k] = s * scale;
                    mx = std::fmax(mx, p[k]);
                }
                float sum = 0.f;
                for (int k = 0; k < T; k++) {
                    p[k] = std::exp(p[k] - mx);
                    sum += p[k];
                }
                const float inv = 1.0f / sum;
                float* o = &att[(size_t)q * d + hh * dk];
                for (int i = 0; i < dk; i++) o[i] = 0.f;
                for (int k = 0; k < T; k++) {
                    const float w = p[k] * inv;
                    const float* vv = &qkv[(size_t)k * 3 * d + 2 * d + hh * dk];
                    for (int i = 0; i < dk; i++) o[i] += w * vv[i];
                }
            }
        });
        linear(att.data(), T, d, L.wout_t, L.bout, d, tmp.data());
        for (size_t i = 0; i < X.size(); i++) X[i] += tmp[i];
        rms_norm(X.data(), L.n2, T, d, h.data());
        linear(h.data(), T, d, L.wgate_t, L.bgate, ff, gu.data());
        linear(h.data(), T, d, L.wup_t, L.bup, ff, uu.data());
        for (size_t i = 0; i < gu.size(); i++) {
            const float g = gu[i];
            gu[i] = (g / (1.0f + std::exp(-g))) * uu[i];
        }
        linear(gu.data(), T, ff, L.wdown_t, L.bdown, d, tmp.data());
        for (size_t i = 0; i < X.size(); i++) X[i] += tmp[i];
    }
    std::vector<float> P((size_t)T * m.up * d);
    linear(X.data(), T, d, m.wupp_t, m.bupp, m.up * d, P.data());  // [T][up*d] == [T*up][d]
    logits.assign((size_t)T * m.up * m.n_phones, 0.f);
    linear(P.data(), T * m.up, d, m.whead_t, m.bhead, m.n_phones, logits.data());
}

}  // namespace

extern "C" {

// Parses a G2P3 blob (src/g2p.h:442-640); nullptr and a message on error.
void* og2p_load(const uint8_t* blob, size_t n, char* err, size_t err_cap) {
    auto fail = [&](const char* m) -> void* {
        if (err && err_cap) std::snprintf(err, err_cap, "%s", m);
        return nullptr;
    };
    if (n < 44 || std::memcmp(blob, "G2P3", 4) != 0) return fail("expected G2P3 format");
    Reader r{blob, n, 4};
    uint32_t hdr[10];
    for (auto& v : hdr) r.u32(v);
    G2P* m = new G2P;
    m->d = (int)hdr[0]; m->heads = (int)hdr[1]; m->n_layers = (int)hdr[2]; m->ff = (int)hdr[3];
    m->up = (int)hdr[4]; m->n_chars = (int)hdr[5]; m->n_phones = (int)hdr[6];
    const uint32_t flags = hdr[9];
    if ((flags & 2) || (flags & 4)) { delete m; return fail("QK-Norm and ConvModule not supported"); }
    if (!(flags & 8)) { delete m; return fail("only RMSNorm supported"); }
    if (m->heads <= 0 || m->d % m->heads) { delete m; return fail("bad head count"); }
    m->dk = m->d / m->heads;
    uint32_t cnt = 0;
    if (!r.u32(cnt)) { delete m; return fail("truncated"); }
    for (uint32_t i = 0; i < cnt; i++) {
        uint32_t cp, id;
        if (!r.u32(cp) || !r.u32(id)) { delete m; return fail("truncated"); }
        m->char2id[cp] = (int)id;
    }
    if (!r.u32(cnt)) { delete m; return fail("truncated"); }
    for (uint32_t i = 0; i < cnt; i++) {
        uint32_t cp, id;
        if (!r.u32(cp) || !r.u32(id)) { delete m; return fail("truncated"); }
        m->id2phone[(int)id] = cp;
    }
    const int d = m->d, ff = m->ff;
    std::vector<float> w;
    bool ok = r.f32(m->emb, (size_t)m->n_chars * d);
    m->layers.resize(m->n_layers);
    for (Layer& L : m->layers) {
        ok = ok && r.f32(L.n1, d);
        ok = ok && r.f32(w, (size_t)3 * d * d); if (ok) L.wqkv_t = transpose(w.data(), 3 * d, d);
        ok = ok && r.f32(L.bqkv, 3 * d);
        ok = ok && r.f32(w, (size_t)d * d); if (ok) L.wout_t = transpose(w.data(), d, d);
        ok = ok && r.f32(L.bout, d);
        ok = ok && r.f32(L.n2, d);
        ok = ok && r.f32(w, (size_t)ff * d); if (ok) L.wgate_t = transpose(w.data(), ff, d);
        ok = ok && r.f32(L.bgate, ff);
        ok = ok && r.f32(w, (size_t)ff * d); if (ok) L.wup_t = transpose(w.data(), ff, d);
        ok = ok && r.f32(L.bup, ff);
        ok = ok && r.f32(w, (size_t)d * ff); if (ok) L.wdown_t = transpose(w.data(), d, ff);
        ok = ok && r.f32(L.bdown, d);
    }
    ok = ok && r.f32(w, (size_t)m->up * d * d); if (ok) m->wupp_t = transpose(w.data(), m->up * d, d);
    ok = ok && r.f32(m->bupp, (size_t)m->up * d);
    ok = ok && r.f32(w, (size_t)m->n_phones * d); if (ok) m->whead_t = transpose(w.data(), m->n_phones, d);
    ok = ok && r.f32(m->bhead, m->n_phones);
    if (!ok) { delete m; return fail("truncated weights"); }
    // RoPE tables exactly as the reference computes them (float pow / cos / sin)
    const int d2 = m->dk / 2;
    m->rope_cos.assign((size_t)G2P::kMaxPos * d2, 0.f);
    m->rope_sin.assign((size_t)G2P::kMaxPos * d2, 0.f);
    if (flags & 1)
        for (int t = 0; t < G2P::kMaxPos; t++)
            for (int i = 0; i < d2; i++) {
                const float freq = (float)t / std::pow(10000.0f, (float)(2 * i) / m->dk);
                m->rope_cos[(size_t)t * d2 + i] = std::cos(freq);
                m->rope_sin[(size_t)t * d2 + i] = std::sin(freq);
            }
    return m;
}

void og2p_free(void* h) { delete static_cast<G2P*>(h); }

// d, heads, n_layers, ff, up, n_chars, n_phones
void og2p_dims(void* h, int* out7) {
    const G2P* m = static_cast<G2P*>(h);
    const int v[7] = {m->d, m->heads, m->n_layers, m->ff, m->up, m->n_chars, m->n_phones};
    std::memcpy(out7, v, sizeof v);
}

// The input's char ids (unknown code points -> 0); returns the count or -1 if cap is short.
int og2p_ids(void* h, const char* text, size_t bytes, int32_t* ids, size_t cap) {
    const G2P* m = static_cast<G2P*>(h);
    std::vector<uint32_t> cps = codepoints(text, bytes);
    if (cps.size() > cap) return -1;
    for (size_t i = 0; i < cps.size(); i++) {
        auto it = m->char2id.find(cps[i]);
        ids[i] = it != m->char2id.end() ? it->second : 0;
    }
    return (int)cps.size();
}

// Forward pass of one text: logits [T*up][n_phones] (if non-null) and argmax ids [T*up].
// Returns T*up, 0 for an empty or over-long (> 2048 characters) input, -1 if a cap is short.
long og2p_forward(void* h, const char* text, size_t bytes, float* logits, size_t logits_cap, int32_t* best,
                  size_t best_cap) {
    const G2P* m = static_cast<G2P*>(h);
    std::vector<int32_t> ids(bytes + 1);
    const int T = og2p_ids(h, text, bytes, ids.data(), ids.size());
    if (T <= 0 || T > G2P::kMaxPos) return 0;
    ids.resize(T);
    std::vector<int> idv(ids.begin(), ids.end());
    std::vector<float> lg;
    forward(*m, idv, lg);
    const long rows = (long)T * m->up;
    if ((size_t)rows > best_cap || (logits && lg.size() > logits_cap)) return -1;
    if (logits) std::memcpy(logits, lg.data(), lg.size() * 4);
    for (long r = 0; r < rows; r++) {
        const float* row = &lg[(size_t)r * m->n_phones];
        int b = 0;
        float bv = row[0];
        for (int c = 1; c < m->n_phones; c++)
            if (row[c] > bv) { bv = row[c]; b = c; }
        best[r] = b;
    }
    return rows;
}

// CTC collapse of per-frame ids to UTF-8 phones (src/g2p.h:865-882); returns bytes or -1 if cap is short.
long og2p_ctc(void* h, const int32_t* best, long rows, char* out, size_t cap) {
    const G2P* m = static_cast<G2P*>(h);
    std::string s;
    int prev = -1;
    for (long t = 0; t < rows; t++) {
        const int b = best[t];
        if (b != 0 && b != prev) {
            auto it = m->id2phone.find(b);
            if (it != m->id2phone.end()) put_utf8(s, it->second);
        }
        prev = b;
    }
    if (s.size() > cap) return -1;
    std::memcpy(out, s.data(), s.size());
    return (long)s.size();
}

}  // extern "C"
