// enc_stack.h -- the Qwen3 encoder stack of qwen3_enc.cpp as a building block for the models that
// run one over projected inputs instead of token ids: the lyric and timbre encoders
// (src/cond-enc.h) and the FSQ tokenizer / detokenizer (src/fsq-tok.h, src/fsq-detok.h).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/acb_models.h"
#include "gguf.h"

namespace acb {

// Load the layers `prefix`layers.{i}.* and `prefix`norm.weight (and `prefix`embed_tokens.weight
// when with_embed) with config cfg; window > 0 on a bidirectional stack masks the even layers to
// |i - j| <= window (cond-enc.h:203-208).
acb_status enc_stack_load(GGUFFile & gf, const std::string & prefix, const acb_qwen3_config & cfg, int window,
                          bool with_embed, int device, acb_qwen3_enc ** out);
// Size the scratch for B sequences of S rows (positions 0..S-1 in each) and return the stack's
// input buffer, f32 [B*S][hidden], for the caller's producer to fill on stream s (nullptr on
// failure). Synchronises s first.
float * enc_stack_input(acb_qwen3_enc * m, int B, int S, cudaStream_t s);
// Every layer, then the final RMSNorm into d_out (rows ldo floats apart), enqueued on s.
acb_status enc_stack_run(acb_qwen3_enc * m, int B, int S, float * d_out, int64_t ldo, cudaStream_t s);
// The stack's device error flag (ACB_DEVERR_* bits of its kernels).
int * enc_stack_err(acb_qwen3_enc * m);

}  // namespace acb
