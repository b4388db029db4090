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
rk_status enqueue_decode(rk_ctx* c, int L);
}  // namespace rk
