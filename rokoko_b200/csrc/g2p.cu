// g2p.cu -- the neural phonemizer (rokoko::G2PModelCuda, src/g2p.h) on B200:
// text -> per-character ids -> G2P3 Conformer-CTC -> IPA, for many texts per call.
//
// The reference phonemizes one text per call with TF32 CUTLASS GEMMs and
// SIMT kernels (src/g2p.h:678-882).  Here every linear layer of every text of
// a call runs as one tcgen05 launch over all texts' rows (texts packed back to
// back; FP32 semantics: split-bf16 products, FP32 accumulate; biases and the
// residual adds in the conv epilogue), attention runs per (text, head) in one
// tcgen05 launch (attention_tc: S and E V in TMEM, online softmax beyond 512
// characters), and the small row kernels below fuse what lies between the
// GEMMs: the char-embedding gather with the first RMSNorm, RMSNorm with the
// 16-bit operand pack, RoPE in place on Q and K, SwiGLU with the pack of the
// down projection, and the per-frame argmax.  The host reads the per-frame ids
// back once per call and collapses them per text (CTC).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_bf16.h>

#include "../../include/rk_b200.h"
#include "conv_tc.cuh"
#include "exec.h"
#include "front_ops.cuh"
#include "g2p.h"
#include "status.h"

namespace rk {

namespace {

// ------------------------------------------------------------------ kernels

// 8 FP32 values -> one 16-byte chunk of the bf16 hi and lo planes
__device__ __forceinline__ void store8_split(void* hi, void* lo, size_t e, const float (&v)[8]) {
    __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        h[j] = __float2bfloat16_rn(v[j]);
        l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
    }
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(hi) + e) = *reinterpret_cast<uint4*>(h);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(lo) + e) = *reinterpret_cast<uint4*>(l);
}

// One warp per row: x_row = ids ? table[ids[r]] : x[r] (written to x_out when
// given: the embedding gather); out = w * x_row / sqrt(mean(x_row^2) + 1e-6)
// (src/g2p.h:55-80) into the operand planes [R][d].  d is a multiple of 8.
__global__ void g2p_rms_pack_kernel(const float* __restrict__ x, const int* __restrict__ ids,
                                    float* __restrict__ x_out, const float* __restrict__ w, int R, int d,
                                    void* hi, void* lo) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= R) return;
    const float* src = x + (size_t)(ids ? ids[row] : row) * d;
    constexpr int MAXV = 4;  // up to 4 x 256 = 1024 columns per row in registers
    float v[MAXV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < MAXV; k++) {
        const int c = (k * 32 + lane) * 8;
        if (c < d) {
            const float4 a = reinterpret_cast<const float4*>(src + c)[0], b = reinterpret_cast<const float4*>(src + c)[1];
            v[k][0] = a.x; v[k][1] = a.y; v[k][2] = a.z; v[k][3] = a.w;
            v[k][4] = b.x; v[k][5] = b.y; v[k][6] = b.z; v[k][7] = b.w;
#pragma unroll
            for (int j = 0; j < 8; j++) ss += v[k][j] * v[k][j];
            if (x_out) {
                reinterpret_cast<float4*>(x_out + (size_t)row * d + c)[0] = a;
                reinterpret_cast<float4*>(x_out + (size_t)row * d + c)[1] = b;
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)d + 1e-6f);
#pragma unroll
    for (int k = 0; k < MAXV; k++) {
        const int c = (k * 32 + lane) * 8;
        if (c < d) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; j++) o[j] = w[c + j] * v[k][j] * inv;
            store8_split(hi, lo, (size_t)row * d + c, o);
        }
    }
}

// RoPE in place on the Q and K parts of QKV rows [R][3d] (src/g2p.h:171-205):
// per head, (x_i, x_{i + dk/2}) -> (x_i cos - x_{i+dk/2} sin, x_{i+dk/2} cos + x_i sin)
// at the row's position within its text.
__global__ void g2p_rope_kernel(float* __restrict__ qkv, const int* __restrict__ pos,
                                const float* __restrict__ cosb, const float* __restrict__ sinb, int R, int d,
                                int heads) {
    const int d2 = d / heads / 2, per_row = 2 * heads * d2;
    const long total = (long)R * per_row;
    for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const int r = (int)(idx / per_row);
        int k = (int)(idx - (long)r * per_row);
        const int part = k / (heads * d2);  // 0: Q, 1: K
        k -= part * heads * d2;
        const int h = k / d2, i = k - h * d2;
        const int p = pos[r];
        float* b = qkv + (size_t)r * 3 * d + part * d + h * 2 * d2;
        const float c = cosb[(size_t)p * d2 + i], s = sinb[(size_t)p * d2 + i];
        const float x0 = b[i], x1 = b[d2 + i];
        b[i] = x0 * c - x1 * s;
        b[d2 + i] = x1 * c + x0 * s;
    }
}

// SwiGLU (src/g2p.h:144-156; the biases are already in): out = g / (1 + e^-g) * u
// for rows [R][gate ff | up ff], packed into the planes [R][ff].  One thread = 8 columns.
__global__ void g2p_swiglu_pack_kernel(const float* __restrict__ gu, int R, int ff, void* hi, void* lo) {
    const int groups = ff / 8;
    const long total = (long)R * groups;
    for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const int r = (int)(idx / groups), c = (int)(idx - (long)r * groups) * 8;
        const float* g = gu + (size_t)r * 2 * ff + c;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float gv = g[j], uv = g[ff + j];
            o[j] = (gv / (1.0f + expf(-gv))) * uv;
        }
        store8_split(hi, lo, (size_t)r * ff + c, o);
    }
}

// Per-frame argmax over the phone logits (bias already in), the first maximum
// on ties (src/g2p.h:353-366).  One warp per row.
__global__ void g2p_argmax_kernel(const float* __restrict__ logits, int rows, int n, int* __restrict__ best) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = logits + (size_t)row * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < n; c += 32) {
        const float v = x[c];
        if (v > bv || (bi == 0x7fffffff)) { bv = v; bi = c; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) best[row] = bi;
}

int grid_for(long work, int threads) {
    long b = (work + threads - 1) / threads;
    if (b > 148L * 16) b = 148L * 16;
    return (int)(b < 1 ? 1 : b);
}

// ------------------------------------------------------------------ weights

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct HostImage {  // 256-byte aligned slices of one host buffer, uploaded as one allocation
    std::vector<uint8_t> bytes;
    size_t put(const void* p, size_t n) {
        const size_t off = al256(bytes.size());
        bytes.resize(off + n, 0);
        if (n) std::memcpy(bytes.data() + off, p, n);
        return off;
    }
};

// a Linear [out][in] as a K = 1 conv: bf16 hi / lo planes [rows padded to 128][Cp]
struct PendingLinear {
    ConvW* w;
    size_t hi, lo, bias;
};

void add_linear(HostImage& img, std::vector<PendingLinear>& todo, ConvW& cw, const float* w, const float* b, int out,
                int in) {
    cw = ConvW{};
    cw.C_in = in; cw.C_out = out; cw.K = 1; cw.taps = 1; cw.Cp = (in + 63) / 64 * 64; cw.phases = 1;
    cw.split = true;
    const size_t rows = (size_t)conv_tc_weight_rows(out);
    std::vector<__nv_bfloat16> h(rows * cw.Cp, __float2bfloat16_rn(0.f)), l(rows * cw.Cp, __float2bfloat16_rn(0.f));
    for (int o = 0; o < out; o++)
        for (int i = 0; i < in; i++) {
            const float v = w[(size_t)o * in + i];
            const __nv_bfloat16 hv = __float2bfloat16_rn(v);
            h[(size_t)o * cw.Cp + i] = hv;
            l[(size_t)o * cw.Cp + i] = __float2bfloat16_rn(v - __bfloat162float(hv));
        }
    PendingLinear p{&cw, img.put(h.data(), h.size() * 2), img.put(l.data(), l.size() * 2),
                    img.put(b, (size_t)out * 4)};
    todo.push_back(p);
}

struct Reader {
    const uint8_t* p;
    size_t n, off;
    bool u32(uint32_t& v) {
        if (off + 4 > n) return false;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return true;
    }
    const float* f32(size_t cnt) {  // view into the blob (unaligned reads copied by the caller)
        if (off + 4 * cnt > n) return nullptr;
        const float* r = reinterpret_cast<const float*>(p + off);
        off += 4 * cnt;
        return r;
    }
};

std::vector<float> copy_f32(const float* p, size_t n) {
    std::vector<float> v(n);
    std::memcpy(v.data(), p, n * 4);
    return v;
}

rk_status load_g2p(rk_ctx* c, const uint8_t* blob, size_t n) {
    // src/g2p.h:442-640: magic, header, vocabularies, FP32 weights in file order
    if (n < 48 || std::memcmp(blob, "G2P3", 4) != 0) return fail(RK_ERR_WEIGHTS, "G2P: expected G2P3 format");
    // the kernels' shared-memory opt-ins (a context may hold a G2P model and no TTS weights)
    if (conv_tc_init() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "conv kernel attributes");
    if (attention_tc_init() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "attention kernel attributes");
    Reader r{blob, n, 4};
    uint32_t hdr[10];
    for (auto& v : hdr) r.u32(v);
    G2PState* s = new G2PState;
    G2PW& m = s->w;
    auto bad = [&](const char* what) { delete s; return fail(RK_ERR_WEIGHTS, what); };
    m.d = (int)hdr[0]; m.heads = (int)hdr[1]; m.n_layers = (int)hdr[2]; m.ff = (int)hdr[3]; m.up = (int)hdr[4];
    m.n_chars = (int)hdr[5]; m.n_phones = (int)hdr[6];
    const uint32_t flags = hdr[9];
    if ((flags & 2) || (flags & 4)) return bad("G2P: QK-Norm and ConvModule not supported");
    if (!(flags & 8)) return bad("G2P: only RMSNorm supported (got LayerNorm model)");
    if (m.heads < 1 || m.d != 64 * m.heads || m.d > 1024 || m.ff % 64 || m.ff < 64 || m.up < 1 ||
        m.n_layers < 1 || m.n_chars < 1 || m.n_phones < 1)
        return bad("G2P: unsupported dimensions (this build needs head_dim 64, d <= 1024, ff % 64 == 0)");
    uint32_t cnt = 0;
    if (!r.u32(cnt)) return bad("G2P: truncated");
    for (uint32_t i = 0; i < cnt; i++) {
        uint32_t cp, id;
        if (!r.u32(cp) || !r.u32(id)) return bad("G2P: truncated");
        if ((int)id >= m.n_chars) return bad("G2P: char id outside the embedding");
        m.char2id[cp] = (int)id;
    }
    if (!r.u32(cnt)) return bad("G2P: truncated");
    for (uint32_t i = 0; i < cnt; i++) {
        uint32_t cp, id;
        if (!r.u32(cp) || !r.u32(id)) return bad("G2P: truncated");
        m.id2phone[(int)id] = cp;
    }
    const int d = m.d, ff = m.ff;
    HostImage img;
    std::vector<PendingLinear> todo;
    const float* emb = r.f32((size_t)m.n_chars * d);
    if (!emb) return bad("G2P: truncated weights");
    const size_t emb_off = img.put(emb, (size_t)m.n_chars * d * 4);
    m.layers.resize(m.n_layers);
    std::vector<size_t> n1_off(m.n_layers), n2_off(m.n_layers);
    size_t params = (size_t)m.n_chars * d;
    for (int li = 0; li < m.n_layers; li++) {
        G2PLayerW& L = m.layers[li];
        const float *n1 = r.f32(d), *qw = r.f32((size_t)3 * d * d), *qb = r.f32(3 * d), *ow = r.f32((size_t)d * d),
                    *ob = r.f32(d), *n2 = r.f32(d), *gw = r.f32((size_t)ff * d), *gb = r.f32(ff),
                    *uw = r.f32((size_t)ff * d), *ub = r.f32(ff), *dw = r.f32((size_t)d * ff), *db = r.f32(d);
        if (!db) return bad("G2P: truncated weights");
        n1_off[li] = img.put(n1, d * 4);
        n2_off[li] = img.put(n2, d * 4);
        std::vector<float> qwv = copy_f32(qw, (size_t)3 * d * d), qbv = copy_f32(qb, 3 * d);
        add_linear(img, todo, L.qkv, qwv.data(), qbv.data(), 3 * d, d);
        std::vector<float> owv = copy_f32(ow, (size_t)d * d), obv = copy_f32(ob, d);
        add_linear(img, todo, L.out, owv.data(), obv.data(), d, d);
        // gate and up stacked into one [2 ff][d] linear: rows [gate | up] (src/g2p.h:596-607)
        std::vector<float> guw((size_t)2 * ff * d), gub(2 * ff);
        std::memcpy(guw.data(), gw, (size_t)ff * d * 4);
        std::memcpy(guw.data() + (size_t)ff * d, uw, (size_t)ff * d * 4);
        std::memcpy(gub.data(), gb, ff * 4);
        std::memcpy(gub.data() + ff, ub, ff * 4);
        add_linear(img, todo, L.gate_up, guw.data(), gub.data(), 2 * ff, d);
        std::vector<float> dwv = copy_f32(dw, (size_t)d * ff), dbv = copy_f32(db, d);
        add_linear(img, todo, L.down, dwv.data(), dbv.data(), d, ff);
        params += 2 * (size_t)d + 3 * (size_t)d * d + 3 * d + (size_t)d * d + d + 3 * (size_t)ff * d + 2 * ff + d;
    }
    const float *upw = r.f32((size_t)m.up * d * d), *upb = r.f32((size_t)m.up * d), *hw = r.f32((size_t)m.n_phones * d),
                *hb = r.f32(m.n_phones);
    if (!hb) return bad("G2P: truncated weights");
    if (r.off != n) return bad("G2P: trailing bytes after the weights");
    {
        std::vector<float> a = copy_f32(upw, (size_t)m.up * d * d), b = copy_f32(upb, (size_t)m.up * d);
        add_linear(img, todo, m.upw, a.data(), b.data(), m.up * d, d);
        std::vector<float> e = copy_f32(hw, (size_t)m.n_phones * d), f = copy_f32(hb, m.n_phones);
        add_linear(img, todo, m.head, e.data(), f.data(), m.n_phones, d);
    }
    params += (size_t)m.up * d * d + (size_t)m.up * d + (size_t)m.n_phones * d + m.n_phones;
    // RoPE tables as the reference computes them on the host (float pow / cos / sin, src/g2p.h:558-568);
    // zeros when the file has no RoPE flag (the rotation is then not applied)
    const int d2 = d / m.heads / 2;
    std::vector<float> rc((size_t)G2P_MAX_POS * d2, 0.f), rs((size_t)G2P_MAX_POS * d2, 0.f);
    if (flags & 1)
        for (int t = 0; t < G2P_MAX_POS; t++)
            for (int i = 0; i < d2; i++) {
                const float freq = (float)t / std::pow(10000.0f, (float)(2 * i) / (float)(d / m.heads));
                rc[(size_t)t * d2 + i] = std::cos(freq);
                rs[(size_t)t * d2 + i] = std::sin(freq);
            }
    const size_t rc_off = img.put(rc.data(), rc.size() * 4), rs_off = img.put(rs.data(), rs.size() * 4);
    void* base = nullptr;
    if (cudaMalloc(&base, std::max<size_t>(img.bytes.size(), 256)) != cudaSuccess) {
        cudaGetLastError();
        delete s;
        return fail(RK_ERR_OOM, "G2P weight allocation");
    }
    m.base = base;
    auto at = [&](size_t off) { return reinterpret_cast<float*>(static_cast<char*>(base) + off); };
    if (cudaMemcpy(base, img.bytes.data(), img.bytes.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(base);
        delete s;
        return fail_cuda(RK_ERR_CUDA, "G2P weight upload");
    }
    m.emb = at(emb_off);
    m.rope_cos = at(rc_off);
    m.rope_sin = at(rs_off);
    for (int li = 0; li < m.n_layers; li++) { m.layers[li].n1 = at(n1_off[li]); m.layers[li].n2 = at(n2_off[li]); }
    for (const PendingLinear& p : todo) {
        ConvW& cw = *p.w;
        cw.hi = at(p.hi); cw.lo = at(p.lo); cw.bias = at(p.bias);
        const uint64_t cols = (uint64_t)cw.Cp, rows = (uint64_t)conv_tc_weight_rows(cw.C_out);
        if (!make_tmap_k64(&cw.tm_hi, cw.hi, true, cols, rows, cols, CONV_W_ROWS) ||
            !make_tmap_k64(&cw.tm_lo, cw.lo, true, cols, rows, cols, CONV_W_ROWS)) {
            cudaFree(base);
            delete s;
            return fail(RK_ERR_INIT, "tensor map encoding failed (G2P weights)");
        }
    }
    m.bytes = params * 4;
    free_g2p(c);
    c->g2p = s;
    return RK_OK;
}

// ------------------------------------------------------------------ workspace

rk_status ensure_g2p_ws(rk_ctx* c, int R, int n) {
    G2PState& s = *c->g2p;
    G2PWS& w = s.ws;
    const G2PW& m = s.w;
    if (w.cap_R >= R && w.cap_n >= n) return RK_OK;
    R = std::max(R, w.cap_R);
    n = std::max(n, w.cap_n);
    if (!w.allocs.empty()) {
        cudaStreamSynchronize(c->stream);
        for (void* p : w.allocs) cudaFree(p);
        w.allocs.clear();
    }
    if (w.h_stage) { cudaFreeHost(w.h_stage); w.h_stage = nullptr; }
    const size_t r = (size_t)R, ru = r * m.up;
    const size_t plane = std::max({r * (size_t)m.ff, ru * (size_t)m.d, r * (size_t)m.d}) * 2;
    struct Req { void** p; size_t bytes; };
    std::vector<Req> reqs = {
        {(void**)&w.meta, (2 * r + 2 * (size_t)n) * 4}, {(void**)&w.x, r * m.d * 4}, {(void**)&w.qkv, r * 3 * m.d * 4},
        {(void**)&w.ctx, r * m.d * 4}, {(void**)&w.gu, r * 2 * m.ff * 4}, {(void**)&w.xu, r * m.up * m.d * 4},
        {(void**)&w.logits, ru * m.n_phones * 4}, {(void**)&w.best, ru * 4}, {&w.op.hi, plane}, {&w.op.lo, plane},
    };
    size_t total = 0;
    for (auto& q : reqs) total += al256(q.bytes);
    char* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        w.cap_R = w.cap_n = 0;
        return fail(RK_ERR_OOM, "G2P workspace allocation");
    }
    w.allocs.push_back(base);
    size_t off = 0;
    for (auto& q : reqs) { *q.p = base + off; off += al256(q.bytes); }
    w.op.plane_bytes = plane;
    w.h_stage_bytes = std::max((2 * r + 2 * (size_t)n) * 4, ru * 4);
    if (cudaMallocHost(&w.h_stage, w.h_stage_bytes) != cudaSuccess) {
        cudaGetLastError();
        w.h_stage = nullptr;
        return fail(RK_ERR_OOM, "G2P pinned staging");
    }
    w.cap_R = R;
    w.cap_n = n;
    return RK_OK;
}

// ------------------------------------------------------------------ forward

void linear(Run& r, const ConvW& w, const Operand& op, int rows, float* y, const float* res = nullptr) {
    ConvCall cc;
    cc.w = &w; cc.op = &op; cc.rows_in = rows; cc.split = true; cc.M = rows; cc.T_out = rows;
    cc.y = y; cc.ldy = w.C_out;
    if (res) { cc.res = res; cc.ldres = w.C_out; }
    cc.no_splitk = true;
    conv(r, cc);
}

// every launch of one call over R rows of n texts (meta already on the device)
void enqueue_g2p(Run& r, G2PState& s, int R, int n, int max_len) {
    const G2PW& m = s.w;
    G2PWS& w = s.ws;
    const int* ids = w.meta;
    const int* pos = w.meta + R;
    SegMeta seg{w.meta + 2 * R, w.meta + 2 * R + n, n, max_len};
    const int warps_grid = (R * 32 + 255) / 256;
    g2p_rms_pack_kernel<<<warps_grid, 256, 0, r.st>>>(m.emb, ids, w.x, m.layers[0].n1, R, m.d, w.op.hi, w.op.lo);
    r.check_launch("g2p_embed_rms_pack");
    for (int li = 0; li < m.n_layers && r.ok(); li++) {
        const G2PLayerW& L = m.layers[li];
        linear(r, L.qkv, w.op, R, w.qkv);
        if (!r.ok()) return;
        g2p_rope_kernel<<<grid_for((long)R * m.d, 256), 256, 0, r.st>>>(w.qkv, pos, m.rope_cos, m.rope_sin, R, m.d,
                                                                       m.heads);
        r.check_launch("g2p_rope");
        cudaError_t e = attention_tc(w.qkv, seg, w.ctx, true, r.c->err, r.st, m.heads);
        r.check_launch("attention_tc");
        if (e != cudaSuccess && r.ok()) r.status = fail_cuda_err(RK_ERR_LAUNCH, "attention_tc", e);
        pack(r, w.ctx, m.d, R, m.d, w.op, m.d, true);
        linear(r, L.out, w.op, R, w.x, w.x);
        if (!r.ok()) return;
        g2p_rms_pack_kernel<<<warps_grid, 256, 0, r.st>>>(w.x, nullptr, nullptr, L.n2, R, m.d, w.op.hi, w.op.lo);
        r.check_launch("g2p_rms_pack");
        linear(r, L.gate_up, w.op, R, w.gu);
        if (!r.ok()) return;
        g2p_swiglu_pack_kernel<<<grid_for((long)R * m.ff / 8, 256), 256, 0, r.st>>>(w.gu, R, m.ff, w.op.hi, w.op.lo);
        r.check_launch("g2p_swiglu_pack");
        linear(r, L.down, w.op, R, w.x, w.x);
        if (!r.ok()) return;
        if (li + 1 < m.n_layers) {
            g2p_rms_pack_kernel<<<warps_grid, 256, 0, r.st>>>(w.x, nullptr, nullptr, m.layers[li + 1].n1, R, m.d,
                                                               w.op.hi, w.op.lo);
            r.check_launch("g2p_rms_pack");
        }
    }
    // upsample: [R][up d] is the memory of [R up][d] (src/g2p.h:337-351), then the head
    pack(r, w.x, m.d, R, m.d, w.op, m.d, true);
    linear(r, m.upw, w.op, R, w.xu);
    pack(r, w.xu, m.d, R * m.up, m.d, w.op, m.d, true);
    linear(r, m.head, w.op, R * m.up, w.logits);
    if (!r.ok()) return;
    g2p_argmax_kernel<<<(R * m.up * 32 + 255) / 256, 256, 0, r.st>>>(w.logits, R * m.up, m.n_phones, w.best);
    r.check_launch("g2p_argmax");
}

// the reference's lenient UTF-8 decoder (src/g2p.h:682-694): the lead byte decides the length
void utf8_codepoints(const char* s, size_t n, std::vector<uint32_t>& out) {
    out.clear();
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
        out.push_back(cp);
    }
}

void put_utf8(std::string& s, uint32_t cp) {  // src/g2p.h:872-877
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

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

void free_g2p(rk_ctx* c) {
    if (!c->g2p) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    G2PState* s = c->g2p;
    for (void* p : s->ws.allocs) cudaFree(p);
    if (s->ws.h_stage) cudaFreeHost(s->ws.h_stage);
    if (s->w.base) cudaFree(s->w.base);
    delete s;
    c->g2p = nullptr;
}

}  // namespace rk

using namespace rk;

extern "C" rk_status rk_g2p_load(rk_ctx* c, const void* blob, size_t bytes) {
    if (!c || !blob) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_g2p_load: null argument");
    DeviceGuard g(c->device);
    return load_g2p(c, static_cast<const uint8_t*>(blob), bytes);
}

extern "C" void rk_g2p_free(rk_ctx* c) {
    if (!c) return;
    DeviceGuard g(c->device);
    free_g2p(c);
}

extern "C" size_t rk_g2p_param_bytes(rk_ctx* c) { return c && c->g2p ? c->g2p->w.bytes : 0; }

extern "C" rk_status rk_g2p_infer(rk_ctx* c, const char* const* texts, const size_t* text_bytes, int n, char* out,
                                  size_t out_cap, size_t* out_len) {
    if (!c || n < 0 || (n > 0 && (!texts || !text_bytes || !out_len)))
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_g2p_infer: bad arguments");
    if (!c->g2p) return fail(RK_ERR_STATE, "rk_g2p_infer: no G2P model loaded (rk_g2p_load)");
    DeviceGuard g(c->device);
    G2PState& s = *c->g2p;
    const G2PW& m = s.w;
    // char ids of every text; empty and over-long texts give "" (src/g2p.h:695-696) and take no rows
    std::vector<std::vector<int32_t>> ids(n);
    std::vector<uint32_t> cps;
    std::vector<int> row_off(n, -1), len(n, 0);
    int R = 0;
    for (int i = 0; i < n; i++) {
        utf8_codepoints(texts[i], text_bytes[i], cps);
        if (cps.empty() || (int)cps.size() > G2P_MAX_POS) continue;
        ids[i].resize(cps.size());
        for (size_t k = 0; k < cps.size(); k++) {
            auto it = m.char2id.find(cps[k]);
            ids[i][k] = it != m.char2id.end() ? it->second : 0;
        }
        row_off[i] = R;
        len[i] = (int)cps.size();
        R += len[i];
    }
    // device passes over groups of consecutive texts (bounded workspace and grid: a launch's
    // grid holds at most 65535 texts); per-text results do not depend on the grouping
    constexpr int kGroupTexts = 4096, kGroupRows = 1 << 18;
    s.ws.last_best.assign((size_t)R * m.up, 0);
    for (int i0 = 0; i0 < n;) {
        int i1 = i0, rows_g = 0, texts_g = 0, max_g = 0;
        while (i1 < n && (row_off[i1] < 0 || texts_g == 0 ||
                          (texts_g < kGroupTexts && rows_g + len[i1] <= kGroupRows))) {
            if (row_off[i1] >= 0) { rows_g += len[i1]; texts_g++; max_g = std::max(max_g, len[i1]); }
            i1++;
        }
        if (texts_g > 0) {
            int base = -1;
            for (int i = i0; i < i1 && base < 0; i++) base = row_off[i];
            rk_status st = ensure_g2p_ws(c, rows_g, texts_g);
            if (st) return st;
            G2PWS& w = s.ws;
            int32_t* h = static_cast<int32_t*>(w.h_stage);
            int k = 0;
            for (int i = i0; i < i1; i++) {
                if (row_off[i] < 0) continue;
                const int o = row_off[i] - base;
                for (int t = 0; t < len[i]; t++) { h[o + t] = ids[i][t]; h[rows_g + o + t] = t; }
                h[2 * rows_g + k] = o;
                h[2 * rows_g + texts_g + k] = len[i];
                k++;
            }
            if (cudaMemcpyAsync(w.meta, h, (2 * (size_t)rows_g + 2 * (size_t)texts_g) * 4, cudaMemcpyHostToDevice,
                                c->stream) != cudaSuccess)
                return fail_cuda(RK_ERR_CUDA, "G2P metadata upload");
            Run r{c, c->stream, true};
            enqueue_g2p(r, s, rows_g, texts_g, max_g);
            if (r.status) {
                cudaStreamSynchronize(c->stream);
                return r.status;
            }
            const size_t frames = (size_t)rows_g * m.up;
            if (cudaMemcpyAsync(h, w.best, frames * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
                return fail_cuda(RK_ERR_CUDA, "G2P frame read-back");
            uint32_t e = 0;
            cudaError_t ce = cudaMemcpyAsync(&e, c->err, 4, cudaMemcpyDeviceToHost, c->stream);
            if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->stream);
            if (ce != cudaSuccess) return fail_cuda_err(RK_ERR_CUDA, "G2P device sync", ce);
            if (e) {
                cudaMemsetAsync(c->err, 0, 4, c->stream);
                return fail(RK_ERR_DEVICE_TIMEOUT, "G2P: a device-side wait gave up");
            }
            std::memcpy(s.ws.last_best.data() + (size_t)base * m.up, h, frames * 4);
        }
        i0 = i1;
    }
    // CTC per text (src/g2p.h:865-882): drop blank 0 and repeats, id -> phone -> UTF-8
    size_t used = 0;
    bool short_buf = false;
    std::string str;
    for (int i = 0; i < n; i++) {
        str.clear();
        if (row_off[i] >= 0) {
            const int32_t* b = s.ws.last_best.data() + (size_t)row_off[i] * m.up;
            int prev = -1;
            for (int t = 0; t < len[i] * m.up; t++) {
                const int id = b[t];
                if (id != 0 && id != prev) {
                    auto it = m.id2phone.find(id);
                    if (it != m.id2phone.end()) put_utf8(str, it->second);
                }
                prev = id;
            }
        }
        out_len[i] = str.size();
        if (!short_buf && used + str.size() <= out_cap && (out || str.empty())) {
            if (!str.empty()) std::memcpy(out + used, str.data(), str.size());
            used += str.size();
        } else {
            short_buf = true;
        }
    }
    if (short_buf) return fail(RK_ERR_WORKSPACE, "rk_g2p_infer: output buffer too small (out_len holds the sizes)");
    return RK_OK;
}

extern "C" rk_status rk_g2p_frames(rk_ctx* c, int32_t* ids, size_t cap, size_t* n) {
    if (!c || !n) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_g2p_frames: bad arguments");
    if (!c->g2p) return fail(RK_ERR_STATE, "rk_g2p_frames: no G2P model loaded");
    const std::vector<int32_t>& b = c->g2p->ws.last_best;
    *n = b.size();
    if (ids) {
        if (cap < b.size()) return fail(RK_ERR_WORKSPACE, "rk_g2p_frames: buffer too small");
        std::memcpy(ids, b.data(), b.size() * 4);
    }
    return RK_OK;
}
