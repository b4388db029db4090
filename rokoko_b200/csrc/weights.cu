// weights.cu -- KOKO v1/v2 weight files -> packed device weights of one rk_ctx.
//
// File format and tensor names: src/weights.cpp:35-50 (parse_header),
// :57-314 (name -> tensor binding), :320-494 (v2 FP16 companions),
// :500-564 (header, 4096-aligned data start).  Weight preparation restates
// precompute_weight_norms (src/rokoko.cpp:1305-1417) and the v1 -> v2
// converter (scripts/convert_v2.py:87-105): w = g v / ||v|| per output row,
// FP16 copies for the FP16-weights semantics.
//
// Unlike the reference (NHWC [C_out, K, C_in] copies for CUTLASS plus an
// im2col/col2im path for ConvTranspose1d), every conv here is packed once into
// the tcgen05 kernel's K-major planes:
//   Conv1d          [C_out][K][Cp]                   Cp = round_up(C_in, 64)
//   strided Conv1d  super-rows [C_out][ceil(K/s)][round_up(s*C_in, 64)]
//   ConvTranspose1d polyphase [s][C_out][K/s][Cp]    (phase r, tap j <- k = r + j*s)
// FP32 semantics keep two bf16 planes (hi, lo = bf16(w - hi)); FP16 keeps one.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "model.h"
#include "front_ops.cuh"
#include "ops.cuh"
#include "status.h"
#include "weights.h"

namespace rk {

// ------------------------------------------------------------------ parsing
bool KokoFile::parse(const uint8_t* blob, size_t n, std::string& err) {
    if (n < 16) { err = "blob too small"; return false; }
    uint32_t magic;
    uint64_t hlen;
    std::memcpy(&magic, blob, 4);
    std::memcpy(&version, blob + 4, 4);
    std::memcpy(&hlen, blob + 8, 8);
    if (magic != 0x4F4B4F4Bu) { err = "bad KOKO magic"; return false; }
    if (version != 1 && version != 2) { err = "unsupported KOKO version"; return false; }
    if (16 + hlen > n) { err = "truncated header"; return false; }
    const size_t data_start = (16 + hlen + 4095) / 4096 * 4096;
    std::istringstream iss(std::string(reinterpret_cast<const char*>(blob) + 16, hlen));
    std::string line;
    while (std::getline(iss, line)) {
        if (line.empty()) continue;
        std::istringstream ls(line);
        KTensor t;
        std::string name;
        size_t off;
        ls >> name >> off >> t.bytes >> t.dtype;
        int d;
        while (ls >> d) t.shape.push_back(d);
        if ((t.dtype != "fp32" && t.dtype != "fp16") || data_start + off + t.bytes > n) {
            err = "bad tensor entry " + name;
            return false;
        }
        t.data = blob + data_start + off;
        tensors[name] = t;
    }
    return true;
}

const KTensor* KokoFile::find(const std::string& name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
}

std::vector<float> KokoFile::f32(const std::string& name) const {
    const KTensor* t = find(name);
    if (!t) throw WeightError("missing tensor " + name);
    const size_t n = t->bytes / (t->dtype == "fp32" ? 4 : 2);
    std::vector<float> v(n);
    if (t->dtype == "fp32") std::memcpy(v.data(), t->data, n * 4);
    else {
        const __half* h = reinterpret_cast<const __half*>(t->data);
        for (size_t i = 0; i < n; i++) v[i] = __half2float(h[i]);
    }
    return v;
}

// ------------------------------------------------------------------ weight image
// Every device-resident weight byte is assembled in one host image (256-byte
// aligned slices) while the structs are filled with tagged image offsets; the
// image is uploaded with one allocation and one copy and the tagged pointers
// are relocated.  The image together with the structs is also what a KOKO v3
// ("B200 layout") file holds, so loading one is a copy plus tensor-map encoding.
namespace {

constexpr uint64_t kTag = 1ull << 62;  // never a device address; image offsets below 2^62

bool tagged(const void* p) { return (reinterpret_cast<uint64_t>(p) & kTag) != 0; }

}  // namespace

void* Image::put(const void* h, size_t n) {
    const size_t off = (bytes.size() + 255) & ~size_t(255);
    bytes.resize(off + n, 0);
    if (n) std::memcpy(bytes.data() + off, h, n);
    return reinterpret_cast<void*>(kTag | off);
}

namespace {

// Visitors over every device pointer and every packed conv of the weight structs.
template <class F, class T>
void vp(T*& p, F& f) {
    void* v = p;
    f(v);
    p = static_cast<T*>(v);
}
template <class F> void visit(ConvW& w, F& f) { vp(w.hi, f); vp(w.lo, f); vp(w.bias, f); }
template <class F> void visit(AdaINW& a, F& f) { vp(a.norm_w, f); vp(a.norm_b, f); }
template <class F> void visit(StyleFC& s, F& f) { vp(s.w, f); vp(s.b, f); vp(s.out, f); }
template <class F> void visit(ResBlk1dW& b, F& f) {
    visit(b.conv1, f); visit(b.conv2, f); visit(b.conv1x1, f); visit(b.norm1, f); visit(b.norm2, f);
    vp(b.pool_w, f); vp(b.pool_b, f);
}
template <class F> void visit(ResBlock1W& r, F& f) {
    for (int j = 0; j < 3; j++) {
        visit(r.convs1[j], f); visit(r.convs2[j], f); visit(r.adain1[j], f); visit(r.adain2[j], f);
        vp(r.alpha1[j], f); vp(r.alpha2[j], f);
    }
}
template <class F> void visit(LstmW& l, F& f) { visit(l.wih, f); vp(l.whh, f); }
template <class F> void visit(DecoderW& d, F& f) {
    vp(d.f0_conv_w, f); vp(d.f0_conv_b, f); vp(d.n_conv_w, f); vp(d.n_conv_b, f);
    visit(d.asr_res, f); visit(d.encode, f);
    for (auto& b : d.decode) visit(b, f);
    for (auto& u : d.ups) visit(u, f);
    for (auto& n : d.noise_convs) visit(n, f);
    for (auto& n : d.noise_res) visit(n, f);
    for (auto& r : d.resblocks) visit(r, f);
    visit(d.conv_post, f); vp(d.source_w, f); vp(d.source_b, f); visit(d.fc, f);
}
template <class F> void visit(FrontW& F_, F& f) {
    vp(F_.word, f); vp(F_.pos, f); vp(F_.type, f); vp(F_.emb_ln_w, f); vp(F_.emb_ln_b, f);
    visit(F_.proj, f); visit(F_.qkv, f); visit(F_.dense, f); visit(F_.ffn, f); visit(F_.ffn_out, f);
    visit(F_.bert_enc, f);
    vp(F_.attn_ln_w, f); vp(F_.attn_ln_b, f); vp(F_.ffn_ln_w, f); vp(F_.ffn_ln_b, f); vp(F_.te_embed, f);
    for (int i = 0; i < 3; i++) { visit(F_.te_conv[i], f); vp(F_.te_ln_g[i], f); vp(F_.te_ln_b[i], f); }
    visit(F_.te_lstm, f);
    for (auto& l : F_.dur_lstm) visit(l, f);
    visit(F_.dur_final, f); visit(F_.shared, f); visit(F_.dur_proj, f);
    for (int i = 0; i < 3; i++) { visit(F_.f0[i], f); visit(F_.nn[i], f); }
    vp(F_.f0_proj_w, f); vp(F_.f0_proj_b, f); vp(F_.n_proj_w, f); vp(F_.n_proj_b, f);
    visit(F_.fc, f);
}

// every packed conv of the structs (the ones with planes)
template <class G> void each_conv(DecoderW& d, FrontW& F_, bool front, G&& g) {
    std::vector<ConvW*> v;
    auto rb1 = [&](ResBlk1dW& b) { v.push_back(&b.conv1); v.push_back(&b.conv2); v.push_back(&b.conv1x1); };
    auto rb = [&](ResBlock1W& r) { for (int j = 0; j < 3; j++) { v.push_back(&r.convs1[j]); v.push_back(&r.convs2[j]); } };
    v.push_back(&d.asr_res); rb1(d.encode);
    for (auto& b : d.decode) rb1(b);
    for (auto& u : d.ups) v.push_back(&u);
    for (auto& n : d.noise_convs) v.push_back(&n);
    for (auto& n : d.noise_res) rb(n);
    for (auto& r : d.resblocks) rb(r);
    v.push_back(&d.conv_post);
    if (front) {
        for (ConvW* w : {&F_.proj, &F_.qkv, &F_.dense, &F_.ffn, &F_.ffn_out, &F_.bert_enc, &F_.dur_proj}) v.push_back(w);
        for (auto& c : F_.te_conv) v.push_back(&c);
        v.push_back(&F_.te_lstm.wih);
        for (auto& l : F_.dur_lstm) v.push_back(&l.wih);
        v.push_back(&F_.dur_final.wih); v.push_back(&F_.shared.wih);
        for (int i = 0; i < 3; i++) { rb1(F_.f0[i]); rb1(F_.nn[i]); }
    }
    for (ConvW* w : v)
        if (w->hi) g(*w);
}

// One allocation + one copy of the image; tagged pointers -> device addresses; tensor maps.
rk_status upload_image(rk_ctx* c, const Image& img, DecoderW& d, FrontW& F_, bool front) {
    void* base = nullptr;
    if (cudaMalloc(&base, std::max<size_t>(img.bytes.size(), 256)) != cudaSuccess) {
        cudaGetLastError();
        return fail(RK_ERR_OOM, "weight image allocation");
    }
    c->weight_allocs.push_back(base);
    if (cudaMemcpy(base, img.bytes.data(), img.bytes.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "weight image upload");
    const uint64_t n = img.bytes.size();
    bool bad = false;
    auto reloc = [&](void*& p) {
        if (!p) return;
        const uint64_t v = reinterpret_cast<uint64_t>(p);
        if (!(v & kTag) || (v & ~kTag) >= n) { bad = true; return; }
        p = static_cast<char*>(base) + (v & ~kTag);
    };
    visit(d, reloc);
    if (front) visit(F_, reloc);
    if (bad) return fail(RK_ERR_WEIGHTS, "weight image: pointer outside the image");
    bool maps_ok = true;
    each_conv(d, F_, front, [&](ConvW& cw) {
        const uint64_t cols = (uint64_t)cw.taps * cw.Cp;
        const uint64_t rows = (uint64_t)conv_tc_weight_rows(cw.phases * cw.C_out);
        maps_ok = maps_ok && make_tmap_k64(&cw.tm_hi, cw.hi, cw.split, cols, rows, cols, CONV_W_ROWS) &&
                  (!cw.split || make_tmap_k64(&cw.tm_lo, cw.lo, true, cols, rows, cols, CONV_W_ROWS));
        if (!cw.split) cw.tm_lo = cw.tm_hi;
    });
    if (!maps_ok) return fail(RK_ERR_INIT, "tensor map encoding failed (weights)");
    c->weights_base = base;
    c->weights_bytes = n;
    return RK_OK;
}

// ------------------------------------------------------------------ KOKO v3 ("B200 layout")
// [u32 magic KOKO][u32 version 3][u64 descriptor bytes]
// descriptor: u32 precision | u32 has_front | u32 layout id | u32 0 | u64 sizeof(DecoderW) |
//             u64 sizeof(FrontW) | u64 image bytes | DecoderW | FrontW (pointers as tagged image offsets)
// zero pad to a multiple of 4096, then the image.  The structs are this build's in-memory
// layout, so a v3 file is read only by a library with the same layout id.
constexpr uint32_t kLayoutId = 0x52423301u ^ (uint32_t)(sizeof(ConvW) * 131 + sizeof(DecoderW) * 7 + sizeof(FrontW));

struct V3Desc {
    uint32_t precision, has_front, layout, zero;
    uint64_t dec_bytes, front_bytes, image_bytes;
};

size_t v3_data_start(size_t desc_bytes) { return (16 + desc_bytes + 4095) / 4096 * 4096; }

rk_status load_v3(rk_ctx* c, const uint8_t* blob, size_t n) {
    uint64_t dlen = 0;
    std::memcpy(&dlen, blob + 8, 8);
    V3Desc h{};
    if (dlen < sizeof(V3Desc) || 16 + dlen > n) return fail(RK_ERR_WEIGHTS, "KOKO v3: truncated descriptor");
    std::memcpy(&h, blob + 16, sizeof h);
    if (h.layout != kLayoutId || h.dec_bytes != sizeof(DecoderW) || h.front_bytes != sizeof(FrontW) ||
        dlen != sizeof(V3Desc) + h.dec_bytes + h.front_bytes)
        return fail(RK_ERR_WEIGHTS, "KOKO v3 file written by a library build with another weight layout; "
                                    "re-export it from the v1 / v2 file");
    if ((int)h.precision != c->precision)
        return fail(RK_ERR_WEIGHTS, h.precision == RK_PRECISION_FP16
                                        ? "KOKO v3 file holds FP16 planes; create the context with RK_PRECISION_FP16"
                                        : "KOKO v3 file holds split-bf16 planes; create the context with RK_PRECISION_FP32");
    const size_t start = v3_data_start(dlen);
    if (start + h.image_bytes > n) return fail(RK_ERR_WEIGHTS, "KOKO v3: truncated image");
    Image img;
    img.bytes.assign(blob + start, blob + start + h.image_bytes);
    std::memcpy(&c->dec, blob + 16 + sizeof(V3Desc), sizeof(DecoderW));
    if (h.has_front) std::memcpy(&c->front, blob + 16 + sizeof(V3Desc) + sizeof(DecoderW), sizeof(FrontW));
    c->has_front = h.has_front != 0;
    return upload_image(c, img, c->dec, c->front, c->has_front);
}

}  // namespace

// ------------------------------------------------------------------ loader
namespace {

float f16_round(float x) { return __half2float(__float2half_rn(x)); }

struct Loader {
    Image& img;
    DecoderW& dec;
    FrontW& front;
    const KokoFile& f;
    bool split;   // FP32 semantics (bf16 hi/lo planes)
    bool v2;      // file holds pre-baked FP16 weights

    // every device-resident byte of the weights goes into one host image; the
    // returned pointer is the image offset tagged (relocated after the upload)
    void* dev_upload(const void* h, size_t bytes) { return img.put(h, bytes); }
    float* dev_f32(const std::vector<float>& v) { return static_cast<float*>(dev_upload(v.data(), v.size() * 4)); }
    float* dev_tensor(const std::string& name) { return dev_f32(f.f32(name)); }

    // Conv weight as [C_out][C_in][K] floats with weight norm applied (v1) or
    // from the v2 FP16 companions; FP16 semantics round to half.
    std::vector<float> conv_weight(const std::string& vname, int Co, int Ci, int K, bool wnorm) {
        std::vector<float> w((size_t)Co * Ci * K);
        if (!v2) {
            std::vector<float> v = f.f32(vname);
            if (v.size() != w.size()) throw WeightError("shape mismatch " + vname);
            if (wnorm) {
                const std::string gname = vname.substr(0, vname.size() - 9) + ".weight_g";
                std::vector<float> g = f.f32(gname);
                const size_t fan = (size_t)Ci * K;
                for (int o = 0; o < Co; o++) {
                    double ss = 0;
                    for (size_t i = 0; i < fan; i++) ss += (double)v[o * fan + i] * v[o * fan + i];
                    const double nrm = std::max(std::sqrt(ss), 1e-12);
                    for (size_t i = 0; i < fan; i++) w[o * fan + i] = (float)((double)g[o] * v[o * fan + i] / nrm);
                }
            } else {
                w = v;
            }
            if (!split)
                for (auto& x : w) x = f16_round(x);
            return w;
        }
        // v2: NHWC fp16 [Co][K][Ci] (possibly C_in padded) or plain fp16 [Co][Ci][K]
        if (const KTensor* t = f.find(vname + ".nhwc_f16")) {
            std::vector<float> n = f.f32(vname + ".nhwc_f16");
            if (n.size() != w.size()) throw WeightError("shape mismatch " + vname);
            for (int o = 0; o < Co; o++)
                for (int k = 0; k < K; k++)
                    for (int i = 0; i < Ci; i++) w[((size_t)o * Ci + i) * K + k] = n[((size_t)o * K + k) * Ci + i];
            (void)t;
            return w;
        }
        for (auto& kv : f.tensors) {
            const std::string pre = vname + ".nhwc_f16_pad";
            if (kv.first.compare(0, pre.size(), pre) == 0) {
                const int cp = std::stoi(kv.first.substr(pre.size()));
                std::vector<float> n = f.f32(kv.first);
                if (n.size() != (size_t)Co * K * cp) throw WeightError("shape mismatch " + kv.first);
                for (int o = 0; o < Co; o++)
                    for (int k = 0; k < K; k++)
                        for (int i = 0; i < Ci; i++) w[((size_t)o * Ci + i) * K + k] = n[((size_t)o * K + k) * cp + i];
                return w;
            }
        }
        if (f.find(vname + ".f16")) {
            std::vector<float> n = f.f32(vname + ".f16");
            if (n.size() != w.size()) throw WeightError("shape mismatch " + vname);
            return n;
        }
        // FP32 tensors kept in v2 (asr_res, F0/N_conv ...): already weight-normed
        if (f.find(vname)) return f.f32(vname);
        throw WeightError("missing tensor " + vname + " (v2)");
    }

    // planes[row][col] <- host floats, converted to bf16 hi/lo or fp16.
    void upload_planes(ConvW& cw, const std::vector<float>& p_in) {
        // rows padded with zeros to a multiple of the kernel's 128-row weight tile
        std::vector<float> p(p_in);
        p.resize((size_t)conv_tc_weight_rows(cw.phases * cw.C_out) * cw.taps * cw.Cp, 0.f);
        const size_t n = p.size();
        if (split) {
            std::vector<__nv_bfloat16> h(n), l(n);
            for (size_t i = 0; i < n; i++) {
                h[i] = __float2bfloat16_rn(p[i]);
                l[i] = __float2bfloat16_rn(p[i] - __bfloat162float(h[i]));
            }
            cw.hi = dev_upload(h.data(), n * 2);
            cw.lo = dev_upload(l.data(), n * 2);
        } else {
            std::vector<__half> h(n);
            for (size_t i = 0; i < n; i++) h[i] = __float2half_rn(p[i]);
            cw.hi = dev_upload(h.data(), n * 2);
            cw.lo = cw.hi;
        }
        cw.split = split;  // tensor maps are encoded after the upload (relocate_and_map)
    }

    // Conv1d (stride 1) from weight [Co][Ci][K] host floats.
    ConvW conv_host(const std::vector<float>& w, int Co, int Ci, int K, const std::vector<float>* bias) {
        ConvW cw;
        cw.C_in = Ci; cw.C_out = Co; cw.K = K; cw.taps = K; cw.Cp = (Ci + 63) / 64 * 64; cw.phases = 1;
        std::vector<float> p((size_t)Co * K * cw.Cp, 0.f);
        for (int o = 0; o < Co; o++)
            for (int i = 0; i < Ci; i++)
                for (int k = 0; k < K; k++) p[((size_t)o * K + k) * cw.Cp + i] = w[((size_t)o * Ci + i) * K + k];
        upload_planes(cw, p);
        if (bias) cw.bias = dev_f32(*bias);
        return cw;
    }

    // Conv1d (stride 1) from weight [Co][Ci][K].
    ConvW conv(const std::string& vname, int Co, int Ci, int K, const char* bias, bool wnorm = true) {
        std::vector<float> w = conv_weight(vname, Co, Ci, K, wnorm);
        std::vector<float> b;
        if (bias) b = f.f32(bias);
        return conv_host(w, Co, Ci, K, bias ? &b : nullptr);
    }

    // Strided Conv1d (dilation 1) re-expressed over super-rows of `s` input rows.
    ConvW conv_strided(const std::string& vname, int Co, int Ci, int K, int s, const char* bias) {
        ConvW cw;
        cw.C_in = Ci; cw.C_out = Co; cw.K = K; cw.stride = s;
        cw.taps = (K + s - 1) / s; cw.Cp = (s * Ci + 63) / 64 * 64; cw.phases = 1;
        std::vector<float> w = conv_weight(vname, Co, Ci, K, false);
        std::vector<float> p((size_t)Co * cw.taps * cw.Cp, 0.f);
        for (int o = 0; o < Co; o++)
            for (int j = 0; j < cw.taps; j++)
                for (int r = 0; r < s; r++) {
                    const int k = j * s + r;
                    if (k >= K) continue;
                    for (int i = 0; i < Ci; i++)
                        p[((size_t)o * cw.taps + j) * cw.Cp + r * Ci + i] = w[((size_t)o * Ci + i) * K + k];
                }
        upload_planes(cw, p);
        if (bias) cw.bias = dev_tensor(bias);
        return cw;
    }

    // ConvTranspose1d weight [Ci][Co][K] (weight norm over dim 0 = C_in) as s
    // polyphase convs with K/s taps: phase r, tap j uses kernel index r + j*s.
    ConvW conv_transpose(const std::string& vname, int Ci, int Co, int K, int s, const char* bias) {
        ConvW cw;
        cw.C_in = Ci; cw.C_out = Co; cw.K = K; cw.phases = s; cw.taps = K / s; cw.Cp = (Ci + 63) / 64 * 64;
        if (K % s) throw WeightError("ConvTranspose1d kernel not a multiple of the stride");
        // conv_weight treats dim 0 as the weight-norm row: here dim 0 = C_in, fan = Co*K
        std::vector<float> w = conv_weight(vname, Ci, Co, K, true);  // [Ci][Co][K]
        std::vector<float> p((size_t)s * Co * cw.taps * cw.Cp, 0.f);
        for (int r = 0; r < s; r++)
            for (int o = 0; o < Co; o++)
                for (int j = 0; j < cw.taps; j++)
                    for (int i = 0; i < Ci; i++)
                        p[(((size_t)r * Co + o) * cw.taps + j) * cw.Cp + i] = w[((size_t)i * Co + o) * K + r + j * s];
        upload_planes(cw, p);
        if (bias) cw.bias = dev_tensor(bias);
        return cw;
    }

    // ---- style FCs
    std::vector<float> fcw, fcb;
    int fc_rows = 0;
    AdaINW adain(const std::string& pf, int C) {
        AdaINW a;
        a.C = C;
        a.norm_w = dev_tensor(pf + ".norm.weight");
        a.norm_b = dev_tensor(pf + ".norm.bias");
        std::vector<float> w = f.f32(v2 ? pf + ".fc.weight.f16" : pf + ".fc.weight");
        std::vector<float> b = f.f32(pf + ".fc.bias");
        if (w.size() != (size_t)2 * C * 128 || b.size() != (size_t)2 * C) throw WeightError("bad fc shape " + pf);
        if (!split && !v2)
            for (auto& x : w) x = f16_round(x);
        a.fc_off = fc_rows;
        fcw.insert(fcw.end(), w.begin(), w.end());
        fcb.insert(fcb.end(), b.begin(), b.end());
        fc_rows += 2 * C;
        return a;
    }
    void finish_fc(StyleFC& fc) {
        fc.rows = fc_rows;
        fc.w = dev_f32(fcw);
        fc.b = dev_f32(fcb);
        fc.out = dev_f32(std::vector<float>((size_t)fc_rows, 0.f));  // per-call output rows
        fcw.clear(); fcb.clear(); fc_rows = 0;
    }

    ResBlk1dW resblk1d(const std::string& pf, int din, int dout, bool shortcut, bool upsample) {
        ResBlk1dW b;
        b.din = din; b.dout = dout; b.shortcut = shortcut; b.upsample = upsample;
        b.norm1 = adain(pf + ".norm1", din);
        b.norm2 = adain(pf + ".norm2", dout);
        b.conv1 = conv(pf + ".conv1.weight_v", dout, din, 3, (pf + ".conv1.bias").c_str());
        b.conv2 = conv(pf + ".conv2.weight_v", dout, dout, 3, (pf + ".conv2.bias").c_str());
        if (shortcut) b.conv1x1 = conv(pf + ".conv1x1.weight_v", dout, din, 1, nullptr);
        if (upsample) {
            // depthwise pool weights stay FP32 (scripts/convert_v2.py:246-248)
            std::vector<float> w((size_t)din * 3);
            if (!v2) {
                std::vector<float> v = f.f32(pf + ".pool.weight_v"), g = f.f32(pf + ".pool.weight_g");
                for (int o = 0; o < din; o++) {
                    double ss = 0;
                    for (int k = 0; k < 3; k++) ss += (double)v[o * 3 + k] * v[o * 3 + k];
                    const double nrm = std::max(std::sqrt(ss), 1e-12);
                    for (int k = 0; k < 3; k++) w[o * 3 + k] = (float)((double)g[o] * v[o * 3 + k] / nrm);
                }
            } else {
                w = f.f32(pf + ".pool.weight_v");
            }
            b.pool_w = dev_f32(w);
            b.pool_b = dev_tensor(pf + ".pool.bias");
        }
        return b;
    }

    ResBlock1W resblock1(const std::string& pf, int C, int K) {
        ResBlock1W r;
        r.C = C; r.K = K;
        for (int j = 0; j < 3; j++) {
            const std::string js = std::to_string(j);
            r.adain1[j] = adain(pf + ".adain1." + js, C);
            r.adain2[j] = adain(pf + ".adain2." + js, C);
            r.convs1[j] = conv(pf + ".convs1." + js + ".weight_v", C, C, K, (pf + ".convs1." + js + ".bias").c_str());
            r.convs2[j] = conv(pf + ".convs2." + js + ".weight_v", C, C, K, (pf + ".convs2." + js + ".bias").c_str());
            r.alpha1[j] = dev_tensor(pf + ".alpha1." + js);
            r.alpha2[j] = dev_tensor(pf + ".alpha2." + js);
        }
        return r;
    }

    // F0_conv / N_conv: Conv1d(1,1,3) with weight norm (FP32 in both files)
    void small_conv(const std::string& pf, float** w, float** b) {
        std::vector<float> v = f.f32(pf + ".weight_v");
        if (!v2) {
            std::vector<float> g = f.f32(pf + ".weight_g");
            double ss = 0;
            for (float x : v) ss += (double)x * x;
            const double nrm = std::max(std::sqrt(ss), 1e-12);
            for (auto& x : v) x = (float)((double)g[0] * x / nrm);
        }
        *w = dev_f32(v);
        *b = dev_tensor(pf + ".bias");
    }

    void load_decoder() {
        DecoderW& d = dec;
        small_conv("decoder.F0_conv", &d.f0_conv_w, &d.f0_conv_b);
        small_conv("decoder.N_conv", &d.n_conv_w, &d.n_conv_b);
        // asr_res stays FP32 in the FP16 variant too (conv1d_f32 with FP32 weights,
        // src/rokoko_f16.cpp:950-952), so it is always packed as split planes.
        {
            const bool keep = split;
            split = true;
            d.asr_res = conv("decoder.asr_res.0.weight_v", 64, 512, 1, "decoder.asr_res.0.bias");
            split = keep;
        }
        d.encode = resblk1d("decoder.encode", 514, 1024, true, false);
        for (int i = 0; i < 4; i++)
            d.decode[i] = resblk1d("decoder.decode." + std::to_string(i), 1090, i < 3 ? 1024 : 512, true, i == 3);
        const std::string g = "decoder.generator";
        d.ups[0] = conv_transpose(g + ".ups.0.weight_v", 512, 256, 20, 10, (g + ".ups.0.bias").c_str());
        d.ups[1] = conv_transpose(g + ".ups.1.weight_v", 256, 128, 12, 6, (g + ".ups.1.bias").c_str());
        d.noise_convs[0] = conv_strided(g + ".noise_convs.0.weight", 256, 22, 12, 6, (g + ".noise_convs.0.bias").c_str());
        d.noise_convs[1] = conv(g + ".noise_convs.1.weight", 128, 22, 1, (g + ".noise_convs.1.bias").c_str(), false);
        d.noise_res[0] = resblock1(g + ".noise_res.0", 256, 7);
        d.noise_res[1] = resblock1(g + ".noise_res.1", 128, 11);
        const int rk_[3] = {3, 7, 11};
        for (int i = 0; i < 6; i++) d.resblocks[i] = resblock1(g + ".resblocks." + std::to_string(i), i < 3 ? 256 : 128, rk_[i % 3]);
        d.conv_post = conv(g + ".conv_post.weight_v", 22, 128, 7, (g + ".conv_post.bias").c_str());
        d.source_w = dev_tensor(g + ".m_source.l_linear.weight");
        d.source_b = dev_tensor(g + ".m_source.l_linear.bias");
        finish_fc(d.fc);
    }

    // Linear layer [out][in] (K = 1 conv)
    ConvW linear(const std::string& wname, int out, int in, const std::string& bname) {
        return conv(wname, out, in, 1, bname.c_str(), false);
    }

    LstmW lstm(const std::string& pf, int in) {
        LstmW l;
        l.in = in;
        std::vector<float> wf = conv_weight(pf + ".weight_ih_l0", 1024, in, 1, false);
        std::vector<float> wr = conv_weight(pf + ".weight_ih_l0_reverse", 1024, in, 1, false);
        wf.insert(wf.end(), wr.begin(), wr.end());
        std::vector<float> bias(2048);
        if (v2) {  // pre-summed bih + bhh (scripts/convert_v2.py:140-146)
            std::vector<float> bf = f.f32(pf + ".bias_combined_fwd"), br = f.f32(pf + ".bias_combined_rev");
            std::copy(bf.begin(), bf.end(), bias.begin());
            std::copy(br.begin(), br.end(), bias.begin() + 1024);
        } else {  // bias = bih + bhh (src/rokoko.cpp:1392-1398)
            std::vector<float> a = f.f32(pf + ".bias_ih_l0"), b = f.f32(pf + ".bias_hh_l0");
            std::vector<float> c = f.f32(pf + ".bias_ih_l0_reverse"), e = f.f32(pf + ".bias_hh_l0_reverse");
            for (int i = 0; i < 1024; i++) { bias[i] = a[i] + b[i]; bias[1024 + i] = c[i] + e[i]; }
        }
        l.wih = conv_host(wf, 2048, in, 1, &bias);
        std::vector<float> hf = conv_weight(pf + ".weight_hh_l0", 1024, 256, 1, false);
        std::vector<float> hr = conv_weight(pf + ".weight_hh_l0_reverse", 1024, 256, 1, false);
        hf.insert(hf.end(), hr.begin(), hr.end());
        l.whh = dev_f32(hf);
        return l;
    }

    int fc_block(const std::string& pf, int rows) {  // plain style FC (AdaLayerNorm): [rows][128] + bias
        std::vector<float> w = f.f32(v2 ? pf + ".fc.weight.f16" : pf + ".fc.weight");
        std::vector<float> b = f.f32(pf + ".fc.bias");
        if (w.size() != (size_t)rows * 128 || b.size() != (size_t)rows) throw WeightError("bad fc shape " + pf);
        if (!split && !v2)
            for (auto& x : w) x = f16_round(x);
        const int off = fc_rows;
        fcw.insert(fcw.end(), w.begin(), w.end());
        fcb.insert(fcb.end(), b.begin(), b.end());
        fc_rows += rows;
        return off;
    }

    void load_front() {
        FrontW& F = front;
        F.word = dev_tensor("bert.embeddings.word_embeddings.weight");
        F.pos = dev_tensor("bert.embeddings.position_embeddings.weight");
        F.type = dev_tensor("bert.embeddings.token_type_embeddings.weight");
        F.emb_ln_w = dev_tensor("bert.embeddings.LayerNorm.weight");
        F.emb_ln_b = dev_tensor("bert.embeddings.LayerNorm.bias");
        F.proj = linear("bert.encoder.embedding_hidden_mapping_in.weight", 768, 128,
                        "bert.encoder.embedding_hidden_mapping_in.bias");
        const std::string a = "bert.encoder.albert_layer_groups.0.albert_layers.0";
        {  // fused Q | K | V projection (three TN+bias GEMMs in the reference, src/rokoko.cpp:356-361)
            std::vector<float> w, b;
            for (const char* n : {"query", "key", "value"}) {
                std::vector<float> wi = conv_weight(a + ".attention." + n + ".weight", 768, 768, 1, false);
                std::vector<float> bi = f.f32(a + ".attention." + n + ".bias");
                w.insert(w.end(), wi.begin(), wi.end());
                b.insert(b.end(), bi.begin(), bi.end());
            }
            F.qkv = conv_host(w, 2304, 768, 1, &b);
        }
        F.dense = linear(a + ".attention.dense.weight", 768, 768, a + ".attention.dense.bias");
        F.attn_ln_w = dev_tensor(a + ".attention.LayerNorm.weight");
        F.attn_ln_b = dev_tensor(a + ".attention.LayerNorm.bias");
        F.ffn = linear(a + ".ffn.weight", 2048, 768, a + ".ffn.bias");
        F.ffn_out = linear(a + ".ffn_output.weight", 768, 2048, a + ".ffn_output.bias");
        F.ffn_ln_w = dev_tensor(a + ".full_layer_layer_norm.weight");
        F.ffn_ln_b = dev_tensor(a + ".full_layer_layer_norm.bias");
        F.bert_enc = linear("bert_encoder.weight", 512, 768, "bert_encoder.bias");
        F.te_embed = dev_tensor("text_encoder.embedding.weight");
        for (int i = 0; i < 3; i++) {
            const std::string pf = "text_encoder.cnn." + std::to_string(i);
            F.te_conv[i] = conv(pf + ".0.weight_v", 512, 512, 5, (pf + ".0.bias").c_str());
            F.te_ln_g[i] = dev_tensor(pf + ".1.gamma");
            F.te_ln_b[i] = dev_tensor(pf + ".1.beta");
        }
        F.te_lstm = lstm("text_encoder.lstm", 512);
        for (int i = 0; i < 3; i++) {
            F.dur_lstm[i] = lstm("predictor.text_encoder.lstms." + std::to_string(2 * i), 640);
            F.aln_off[i] = fc_block("predictor.text_encoder.lstms." + std::to_string(2 * i + 1), 1024);
        }
        F.dur_final = lstm("predictor.lstm", 640);
        F.dur_proj = linear("predictor.duration_proj.linear_layer.weight", 50, 512,
                            "predictor.duration_proj.linear_layer.bias");
        F.shared = lstm("predictor.shared", 640);
        const int din[3] = {512, 512, 256}, dout[3] = {512, 256, 256};
        for (int i = 0; i < 3; i++) {
            F.f0[i] = resblk1d("predictor.F0." + std::to_string(i), din[i], dout[i], i == 1, i == 1);
            F.nn[i] = resblk1d("predictor.N." + std::to_string(i), din[i], dout[i], i == 1, i == 1);
        }
        F.f0_proj_w = dev_tensor("predictor.F0_proj.weight");
        F.f0_proj_b = dev_tensor("predictor.F0_proj.bias");
        F.n_proj_w = dev_tensor("predictor.N_proj.weight");
        F.n_proj_b = dev_tensor("predictor.N_proj.bias");
        finish_fc(F.fc);
    }
};

}  // namespace

void free_weights(rk_ctx* c) {
    for (void* p : c->weight_allocs) cudaFree(p);
    c->weight_allocs.clear();
    c->weights_base = nullptr;
    c->weights_bytes = 0;
    for (auto& p : c->splitk) p = nullptr;  // part of weight_allocs
    c->dec = DecoderW{};
    c->front = FrontW{};
    c->has_front = false;
    c->loaded = false;
}

rk_status build_image(const void* blob, size_t bytes, int precision, Image& img, DecoderW& dec, FrontW& front,
                      bool& has_front) {
    KokoFile f;
    std::string err;
    if (!f.parse(static_cast<const uint8_t*>(blob), bytes, err)) return fail(RK_ERR_WEIGHTS, err.c_str());
    const bool v2 = f.version == 2;
    if (v2 && precision == RK_PRECISION_FP32)
        return fail(RK_ERR_WEIGHTS, "KOKO v2 holds FP16 weights; create the context with RK_PRECISION_FP16");
    try {
        Loader ld{img, dec, front, f, precision == RK_PRECISION_FP32, v2};
        ld.load_decoder();
        // the front half is optional: decoder-only files (and callers) use rk_decode_features
        has_front = f.find("bert.embeddings.word_embeddings.weight") != nullptr;
        if (has_front) ld.load_front();
    } catch (WeightError& e) {
        return fail(RK_ERR_WEIGHTS, e.what());
    }
    return RK_OK;
}

rk_status export_v3(int precision, const Image& img, const DecoderW& dec, const FrontW& front, bool has_front,
                    void* dst, size_t cap, size_t* out_bytes) {
    const size_t dlen = sizeof(V3Desc) + sizeof(DecoderW) + sizeof(FrontW);
    const size_t start = v3_data_start(dlen), total = start + img.bytes.size();
    if (out_bytes) *out_bytes = total;
    if (!dst) return RK_OK;
    if (cap < total) return fail(RK_ERR_WORKSPACE, "rk_export: destination smaller than the v3 file");
    uint8_t* o = static_cast<uint8_t*>(dst);
    std::memset(o, 0, start);
    const uint32_t magic = 0x4F4B4F4Bu, version = 3;
    const uint64_t dl = dlen;
    std::memcpy(o, &magic, 4);
    std::memcpy(o + 4, &version, 4);
    std::memcpy(o + 8, &dl, 8);
    const V3Desc h{(uint32_t)precision, has_front ? 1u : 0u, kLayoutId, 0u, sizeof(DecoderW), sizeof(FrontW),
                   img.bytes.size()};
    std::memcpy(o + 16, &h, sizeof h);
    // the tensor maps are re-encoded when the file is loaded
    DecoderW d = dec;
    FrontW F_ = front;
    auto clear_maps = [](ConvW& cw) { cw.tm_hi = CUtensorMap{}; cw.tm_lo = CUtensorMap{}; };
    each_conv(d, F_, has_front, clear_maps);
    std::memcpy(o + 16 + sizeof h, &d, sizeof d);
    std::memcpy(o + 16 + sizeof h + sizeof d, &F_, sizeof F_);
    std::memcpy(o + start, img.bytes.data(), img.bytes.size());
    return RK_OK;
}

rk_status load_weights(rk_ctx* c, const void* blob, size_t bytes) {
    const uint8_t* b = static_cast<const uint8_t*>(blob);
    uint32_t magic = 0, version = 0;
    if (bytes >= 16) { std::memcpy(&magic, b, 4); std::memcpy(&version, b + 4, 4); }
    free_weights(c);
    rk_status s;
    if (magic == 0x4F4B4F4Bu && version == 3) {
        s = load_v3(c, b, bytes);
    } else {
        Image img;
        bool front = false;
        s = build_image(blob, bytes, c->precision, img, c->dec, c->front, front);
        if (!s) {
            c->has_front = front;
            s = upload_image(c, img, c->dec, c->front, c->has_front);
        }
    }
    if (s) { free_weights(c); return s; }
    for (auto& p : c->splitk) {
        void* d = nullptr;
        if (cudaMalloc(&d, rk_ctx::kSplitKBytes) != cudaSuccess) {
            cudaGetLastError();
            free_weights(c);
            return fail(RK_ERR_OOM, "split-K scratch");
        }
        c->weight_allocs.push_back(d);
        p = static_cast<float*>(d);
    }
    if (upload_twiddles() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "twiddle upload");
    if (conv_tc_init() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "conv kernel attributes");
    if (bilstm_init() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "lstm kernel attributes");
    if (attention_tc_init() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "attention kernel attributes");
    c->loaded = true;
    return RK_OK;
}

}  // namespace rk

// ------------------------------------------------------------------ C ABI: KOKO v3
extern "C" rk_status rk_convert_koko_b200(const void* blob, size_t bytes, int precision, void* dst, size_t cap,
                                          size_t* out_bytes) {
    using namespace rk;
    if (!blob) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_convert_koko_b200: null input");
    if (precision != RK_PRECISION_FP32 && precision != RK_PRECISION_FP16)
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_convert_koko_b200: unknown precision");
    Image img;
    DecoderW dec;
    FrontW front;
    bool has_front = false;
    rk_status s = build_image(blob, bytes, precision, img, dec, front, has_front);
    if (s) return s;
    return export_v3(precision, img, dec, front, has_front, dst, cap, out_bytes);
}
