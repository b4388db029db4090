/* rk_b200.h -- C ABI of the B200-native Kokoro decoder / front-half library.
 *
 * Plain pointers and sizes only; every function returns an rk_status and
 * never exits the process.  All model state lives in an opaque rk_ctx (one
 * per device); separate contexts may be used from separate threads.
 *
 * Reference interfaces each entry point replaces (paths in LokalOptima/rokoko):
 *   rk_conv1d_fprop        cutlass_conv1d_fprop / _f16   src/cutlass_conv.cu:239-313,
 *                          src/cutlass_conv_f16.cu:216-273 (same argument meaning
 *                          and return codes 0 / -1 / -2 / -3 / -4, plus a precision)
 *   rk_conv1d_fprop_f32    cutlass_conv1d_fprop      src/cutlass_conv.cu:238-244
 *   rk_conv1d_fprop_f16    cutlass_conv1d_fprop_f16  src/cutlass_conv_f16.cu:215-221
 *                          (both with the reference's exact argument list, so a
 *                          caller of the CUTLASS seam relinks unchanged)
 *   rk_conv1d_workspace_bytes  cutlass_conv1d_workspace_bytes  src/cutlass_conv.cu:319-330
 *   rk_create + rk_load_weights_koko
 *                          Weights::load + precompute_weight_norms
 *                          src/weights.cpp:500-601, src/rokoko.cpp:1305-1676,
 *                          src/rokoko_f16.cpp:1177-1197 (KOKO v1 and v2 files)
 *   rk_infer               rokoko_infer  src/weights.h:402-405,
 *                          src/rokoko.cpp:829-1297 (tokens + style -> PCM)
 *   rk_decode_features     the decoder/generator half of rokoko_infer,
 *                          src/rokoko.cpp:915-1290 (no separate entry exists
 *                          in the reference; L is used as given, no bucketing)
 *   rk_compute_decode_bytes  compute_decode_bytes  src/rokoko_common.h:160-229
 */
#ifndef RK_B200_H
#define RK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RK_API __attribute__((visibility("default")))
#else
#define RK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int rk_status;
#define RK_OK 0
#define RK_ERR_CANNOT_IMPLEMENT (-1) /* unsupported shape / argument */
#define RK_ERR_WORKSPACE (-2)        /* caller workspace too small */
#define RK_ERR_INIT (-3)             /* descriptor / context set-up failed */
#define RK_ERR_LAUNCH (-4)           /* kernel launch failed */
#define RK_ERR_CUDA (-5)             /* CUDA runtime error (see rk_last_error) */
#define RK_ERR_WEIGHTS (-6)          /* malformed or incomplete KOKO weight file */
#define RK_ERR_DEVICE_TIMEOUT (-7)   /* a bounded device-side wait gave up */
#define RK_ERR_OOM (-8)              /* device allocation failed */
#define RK_ERR_STATE (-9)            /* call out of order (e.g. no weights loaded) */

#define RK_PRECISION_FP32 0 /* FP32 semantics: 3-pass split-bf16 tensor-core products */
#define RK_PRECISION_FP16 1 /* FP16-weights semantics (KOKO v2): fp16 x fp16, fp32 accumulate */

typedef struct rk_ctx rk_ctx;

typedef struct rk_options {
    int precision;  /* RK_PRECISION_* */
    int max_tokens; /* largest T per utterance (<= 512); 0 = 512 */
    int l_bucket;   /* decode-length bucket (reference: 32); 0 = 32, 1 = none */
} rk_options;

RK_API const char* rk_status_string(rk_status s);
/* Human-readable detail of the last error raised on this thread. */
RK_API const char* rk_last_error(void);

/* ---- stateless conv seam -------------------------------------------------
 * y[T_out, C_out] = conv1d(x[T_in, C_in]) with weights w[C_out, K, C_in] (NHWC,
 * as produced by cutlass_reshape_weights), all FP32 device pointers, time-major.
 * If residual != NULL: y = conv + residual (bias ignored, as in the reference);
 * else if bias != NULL: y = conv + bias[C_out]; else y = conv.
 * precision selects the tensor-core path (RK_PRECISION_*).  stride > 1 requires
 * dilation == 1.  Enqueued on `stream` (a cudaStream_t, NULL = legacy default).
 * workspace: device memory of at least rk_conv1d_workspace_size(...) bytes. */
RK_API size_t rk_conv1d_workspace_size(int C_in, int C_out, int T_in, int K, int stride, int padding, int dilation,
                                int precision);
RK_API rk_status rk_conv1d_fprop(const float* x, const float* w, const float* bias, float* y, const float* residual,
                          void* workspace, size_t workspace_bytes, int C_in, int C_out, int T_in, int K, int stride,
                          int padding, int dilation, int precision, void* stream);
/* Synchronises `stream` and reports (and clears) the device error word kept at
 * the start of a conv workspace: RK_OK or RK_ERR_DEVICE_TIMEOUT. */
RK_API rk_status rk_conv1d_check(void* workspace, void* stream);

/* The reference's conv seam, argument for argument (cudaStream_t is passed as
 * void*; `x` and `w` of the _f16 form point at IEEE half data, the reference's
 * `const __half*`).  _f32: FP32 operands with FP32 semantics (three split-bf16
 * tensor-core products per product); _f16: half operands, fp16 products with
 * FP32 accumulation.  bias, residual and y are FP32 in both, as in the
 * reference.  The workspace (the reference passes its float* arena slice) must
 * hold rk_conv1d_workspace_bytes(...) bytes and be 256-byte aligned; its
 * first 4 bytes are the device error word read by rk_conv1d_check. */
RK_API rk_status rk_conv1d_fprop_f32(const float* x, const float* w, const float* bias, float* y,
                                     const float* residual, float* workspace, size_t workspace_bytes, int C_in,
                                     int C_out, int T_in, int K, int stride, int padding, int dilation,
                                     void* stream);
RK_API rk_status rk_conv1d_fprop_f16(const void* x, const void* w, const float* bias, float* y,
                                     const float* residual, float* workspace, size_t workspace_bytes, int C_in,
                                     int C_out, int T_in, int K, int stride, int padding, int dilation,
                                     void* stream);
/* Workspace bytes for either form above (the larger, FP32, requirement). */
RK_API size_t rk_conv1d_workspace_bytes(int C_in, int C_out, int T_in, int K, int stride, int padding,
                                        int dilation);

/* rk_conv1d_fprop without a workspace argument and without any device
 * allocation.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory where they need the convolution (under a
 * host-owned memory pool, on a thread that must not block on the allocator, or
 * within a fixed plugin budget).  Its scratch is one
 * library-owned device array of RK_CONV_STATIC_SCRATCH_BYTES on each GPU that
 * loads the library, kept until the process exits; shapes whose
 * rk_conv1d_workspace_size exceeds it return RK_ERR_WORKSPACE.  The first call
 * on a device looks up the array's address (make it before any stream
 * capture).  All calls share the array: calls that can overlap on one GPU race
 * and must be serialised by the caller.  Same arguments and results as
 * rk_conv1d_fprop otherwise. */
#define RK_CONV_STATIC_SCRATCH_BYTES (32u * 1024u * 1024u)
RK_API rk_status rk_conv1d_fprop_static(const float* x, const float* w, const float* bias, float* y,
                                        const float* residual, int C_in, int C_out, int T_in, int K, int stride,
                                        int padding, int dilation, int precision, void* stream);
/* Synchronises `stream` and reports (and clears) the device error word of the
 * static scratch array: RK_ERR_DEVICE_TIMEOUT when a bounded device-side wait
 * of an rk_conv1d_fprop_static call on this device gave up (its output is then
 * incomplete), else RK_OK.  Call it after the static calls whose result matters;
 * each rk_conv1d_fprop_static call clears the word when it starts. */
RK_API rk_status rk_conv1d_static_check(void* stream);

/* ---- model context ------------------------------------------------------- */
RK_API rk_status rk_create(int device, const rk_options* opts, rk_ctx** out);
RK_API void rk_destroy(rk_ctx* ctx);
/* KOKO v1 (fp32), v2 (pre-baked fp16) or v3 (B200 layout, below) bytes in host memory. */
RK_API rk_status rk_load_weights_koko(rk_ctx* ctx, const void* host_blob, size_t bytes);

/* KOKO v3, the "B200 layout" file (the next step after the reference's v2
 * converter, scripts/convert_v2.py:111-349, and its loader,
 * src/weights.cpp:320-494): every weight already packed the way the kernels
 * read it (K-major 16-bit planes, bf16 hi + lo for precision RK_PRECISION_FP32
 * or fp16 for RK_PRECISION_FP16, weight norm folded in, output rows padded to
 * the 128-row MMA tile, ConvTranspose1d split into its polyphase planes, LSTM
 * biases summed, style FCs concatenated) in one image, so rk_load_weights_koko
 * reads it with one device allocation and one copy.  Converts a v1 or v2 blob
 * on the host (no GPU needed); *out_bytes receives the file size; dst NULL
 * only sizes it.  A v3 file is read by a library build with the same weight
 * layout and by a context of the same precision (else RK_ERR_WEIGHTS). */
RK_API rk_status rk_convert_koko_b200(const void* host_blob, size_t bytes, int precision, void* dst, size_t cap,
                                      size_t* out_bytes);

/* Decoder + generator on given features, host buffers:
 * asr [L, 512], f0 [2L], n [2L], style [128] (acoustic half) -> pcm [600 L]. */
RK_API rk_status rk_decode_features(rk_ctx* ctx, const float* asr, const float* f0, const float* n, const float* style128,
                             int L, float* pcm_out);
/* Same on device buffers, enqueued on ctx's stream; pcm is a device pointer. */
RK_API rk_status rk_decode_features_device(rk_ctx* ctx, const float* d_asr, const float* d_f0, const float* d_n,
                                    const float* d_style128, int L, float* d_pcm);

/* Full forward for one utterance (rokoko_infer): tokens [T] incl. BOS/EOS,
 * style [256] (ref_s), optional dur_override [T].  Writes dur_out [T] (may be
 * NULL), *L_out (frames before bucketing) and min(600 L, pcm_capacity) samples. */
RK_API rk_status rk_infer(rk_ctx* ctx, const int32_t* tokens, int T, const float* style256, const int32_t* dur_override,
                   int32_t* dur_out, int* L_out, float* pcm_out, size_t pcm_capacity, size_t* n_samples);

/* Batched form (rk_encode + rk_decode; the reference has one utterance per
 * rokoko_infer call, src/weights.h:402-405).  rk_encode runs the front half of
 * B utterances: tokens = the B token lists concatenated (T_per_utt[b] each,
 * incl. BOS/EOS), style [B][256], optional dur_override and dur_out laid out
 * like tokens, L_out [B] (nullable).  Each utterance's decoder inputs stay on
 * the device until rk_decode, which decodes every pending utterance in encode
 * order into pcm (600 * L[b] samples each, concatenated; pcm_capacity must
 * hold them all), n_samples [B] (nullable), *B_out (nullable). */
RK_API rk_status rk_encode(rk_ctx* ctx, const int32_t* tokens, const int32_t* T_per_utt, int B, const float* style,
                           const int32_t* dur_override, int32_t* dur_out, int32_t* L_out);
RK_API rk_status rk_decode(rk_ctx* ctx, float* pcm_out, size_t pcm_capacity, size_t* n_samples, int* B_out);

/* Streaming synthesis (TtsPipeline::synthesize_streaming, src/rokoko.h:298-360;
 * the reference runs one chunk after the other): the B utterances (laid out as
 * for rk_encode) are processed in chunks of `chunk`; while the decoder runs
 * chunk k, the front half of chunk k + 1 runs beside it on the context's
 * second stream.  on_pcm(user, index, pcm, n_samples) receives each
 * utterance's PCM in order (pcm is a library buffer, valid during the call);
 * it returns nonzero to go on and 0 to stop, after which rk_synthesize_stream
 * returns RK_OK with nothing pending.  Durations are predicted unless
 * dur_override (like tokens) is given.  No utterance of rk_encode may be
 * pending. */
typedef int (*rk_pcm_fn)(void* user, int index, const float* pcm, size_t n_samples);
RK_API rk_status rk_synthesize_stream(rk_ctx* ctx, const int32_t* tokens, const int32_t* T_per_utt, int B,
                                      const float* style, const int32_t* dur_override, int chunk,
                                      rk_pcm_fn on_pcm, void* user);

/* Neural phonemizer (rokoko::G2PModelCuda, src/g2p.h:374-430; load
 * src/g2p.h:442-640, infer :678-882): UTF-8 text -> IPA phones.  The G2P3
 * model (RoPE + RMSNorm, heads of 64 dimensions) lives in the context beside
 * (or without) its TTS weights and always computes with FP32 semantics.
 * rk_g2p_load parses a G2P3 blob (RK_ERR_WEIGHTS on a malformed or
 * unsupported file) and replaces any model loaded before.  rk_g2p_infer
 * phonemizes n texts (texts[i], text_bytes[i] bytes each) in one pass on the
 * device: the phones of text i are written to out back to back, out_len[i]
 * bytes each; a text that is empty or longer than 2048 characters gives ""
 * (the reference's rule).  When out_cap is short, out_len still receives every
 * size and the call returns RK_ERR_WORKSPACE.  rk_g2p_frames copies the
 * per-frame CTC ids of the last rk_g2p_infer (up * characters per text, texts
 * in order, empty texts taking none; *n = their count; ids may be NULL to ask
 * for the count).  rk_g2p_param_bytes = the model's FP32 parameter bytes. */
RK_API rk_status rk_g2p_load(rk_ctx* ctx, const void* blob, size_t bytes);
RK_API rk_status rk_g2p_infer(rk_ctx* ctx, const char* const* texts, const size_t* text_bytes, int n, char* out,
                              size_t out_cap, size_t* out_len);
RK_API rk_status rk_g2p_frames(rk_ctx* ctx, int32_t* ids, size_t cap, size_t* n);
RK_API size_t rk_g2p_param_bytes(rk_ctx* ctx);
RK_API void rk_g2p_free(rk_ctx* ctx);

/* IPA -> model input (rokoko::to_tokens / chunk_ipa, src/rokoko.h:141-221),
 * host only.  rk_ipa_to_tokens: BOS 0, the token id of every code point of
 * the IPA text that is in the model's vocabulary (others dropped), EOS 0;
 * *count = ids written (or needed: RK_ERR_WORKSPACE when cap is short; ids
 * may be NULL to ask).  rk_ipa_chunks: the text split into pieces of at most
 * 510 code points, after the last . ! ? within the limit, else the last , : ;,
 * else the last space, else at the limit; ends[k] = end byte offset of piece
 * k, *n = piece count (ends may be NULL to ask). */
RK_API rk_status rk_ipa_to_tokens(const char* ipa, size_t bytes, int32_t* ids, size_t cap, size_t* count);
RK_API rk_status rk_ipa_chunks(const char* ipa, size_t bytes, size_t* ends, size_t cap, size_t* n);

/* Stage activations of the last forward (names as the oracle's stage dumps);
 * copies min(count, cap) floats; *count = element count (0 if unknown). */
RK_API rk_status rk_get_stage(rk_ctx* ctx, const char* name, float* host_dst, size_t cap, size_t* count);
/* Turn per-stage capture on/off (off by default; costs device->host copies). */
RK_API rk_status rk_record_stages(rk_ctx* ctx, int on);

/* Number of kernels this library launched on ctx since the last reset. */
RK_API rk_status rk_kernel_count(rk_ctx* ctx, long long* count, int reset);
/* The CUDA stream (cudaStream_t) all of ctx's work is enqueued on. */
RK_API void* rk_stream(rk_ctx* ctx);

/* Profiling.  rk_profile(ctx, mode), mode a set of RK_PROFILE_* bits (1 = the
 * original "on"), makes decodes replay a separate CUDA graph per mode whose
 * timing events are event nodes (each profiled decode must be read back with
 * rk_profile_read / rk_profile_timeline before the next one):
 *   RK_PROFILE_CONV      every tcgen05 conv launch is bracketed by CUDA events
 *                        on its stream; rk_profile_read synchronises and returns
 *                        the summed device time (ms), the summed algorithmic
 *                        FLOPs (2 C_in C_out K T_out; T_in for ConvTranspose1d)
 *                        and the launch count since rk_profile was called.
 *   RK_PROFILE_SERIAL    every launch of the decode goes to the context stream
 *                        (no concurrent lanes), so per-launch times are the
 *                        kernels' own.
 *   RK_PROFILE_TIMELINE  one event node after every launch.  rk_profile_timeline
 *                        synchronises and writes one text line per launch,
 *                        "<stream>\t<name>\t<end ms>", end times relative to the
 *                        start of the decode (stream 0 = context stream, 1 = the
 *                        noise branch, 2-3 = resblock lanes); *len = bytes
 *                        needed (the text is cut at cap - 1 and NUL-terminated);
 *                        a call with a buffer then forgets the marks. */
#define RK_PROFILE_CONV 1
#define RK_PROFILE_SERIAL 2
#define RK_PROFILE_TIMELINE 4
RK_API rk_status rk_profile(rk_ctx* ctx, int mode);
RK_API rk_status rk_profile_read(rk_ctx* ctx, double* conv_ms, double* conv_flops, long long* conv_launches);
RK_API rk_status rk_profile_timeline(rk_ctx* ctx, char* buf, size_t cap, size_t* len);

RK_API size_t rk_compute_decode_bytes(int T, int L);

#ifdef __cplusplus
}
#endif
#endif /* RK_B200_H */
