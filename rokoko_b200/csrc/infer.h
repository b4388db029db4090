// infer.h -- front half of the forward (ALBERT .. F0/N prediction) for a batch.
#pragma once
#include "../../include/rk_b200.h"

struct rk_ctx;

namespace rk {
// Front half of B utterances (tokens concatenated, T_per[b] each incl. BOS/EOS;
// style [B][256]; optional dur_override laid out like tokens).  Writes the
// predicted durations (dur_out, like tokens) and L per utterance (L_out), and
// appends one pending entry per utterance whose decoder inputs live in the
// context's stash.  Synchronous with respect to the duration read-back only.
rk_status encode_batch(rk_ctx* c, const int32_t* tokens, const int32_t* T_per, int B, const float* style,
                       const int32_t* dur_override, int32_t* dur_out, int32_t* L_out, const char* who);
// Marks the stash chunks of `pool` free again (call when none of its utterances is pending).
void stash_reset(rk_ctx* c, int pool = 0);
void free_front_ws(rk_ctx* c);
}  // namespace rk
