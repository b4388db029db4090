// decode.h -- decoder / generator forward of one rk_ctx.
#pragma once
#include "../../include/rk_b200.h"

struct rk_ctx;

namespace rk {
// Allocates (or grows) the decode workspace for up to L frames.
rk_status ensure_decode_ws(rk_ctx* c, int L);
void free_decode_ws(rk_ctx* c);
// Enqueues the decoder + generator for L frames on c->stream; inputs are read
// from the workspace (asr, f0, n, style), the waveform lands in ws.audio.
// gen_only: the generator alone, from the decoder output already in ws.gx.
rk_status enqueue_decode(rk_ctx* c, int L, bool gen_only = false);

// Decoder + generator for `n` pending utterances (rk_encode's stash entries):
// the decoder blocks of all of them in one pass over their segmented frames,
// then one generator graph per utterance; PCM (600 L samples each) to pcm[i]
// (host, may be null).  Enqueued on c->stream.
struct PendingRef {
    int L, L_b;
    const float *asr, *f0, *n, *style;
};
rk_status decode_batch(rk_ctx* c, const PendingRef* p, int n, float* const* pcm);
void free_decode_batch_ws(rk_ctx* c);
}  // namespace rk
