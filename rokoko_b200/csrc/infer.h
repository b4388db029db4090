// infer.h -- front half of the forward (ALBERT .. F0/N prediction).
#pragma once
#include "../../include/rk_b200.h"

struct rk_ctx;

namespace rk {
rk_status ensure_front_tokens(rk_ctx* c);
rk_status ensure_front_frames(rk_ctx* c, int L_b);
void free_front_ws(rk_ctx* c);
// ALBERT, text encoder, duration encoder, durations (inputs fws.tok, fws.style).
rk_status enqueue_encode(rk_ctx* c, int T);
// alignment (fws.dur_use), shared LSTM, F0/N chains -> decoder inputs in c->ws.
rk_status enqueue_predict(rk_ctx* c, int T, int L_b);
}  // namespace rk
