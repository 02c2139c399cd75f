// adapter.h -- LoRA / LoKr merge into staged GGUF weights at load (src/adapter-merge.h).
#pragma once

#include <cuda_runtime.h>

#include "../../include/acb_models.h"
#include "weights.h"

namespace acb {

// Merge the adapter at adapter_path (a PEFT directory, or one safetensors file: ComfyUI LoRA or
// LyCORIS LoKr) with user scale `scale` into the tensors of `staged` (uploaded, in their GGUF
// types), in place on stream st. *n_merged receives the number of weights changed.
// ACB_ERR_FORMAT when no pair or module matches a weight.
acb_status adapter_merge(const char * adapter_path, float scale, WeightArena & staged, cudaStream_t st,
                         int * n_merged);

}  // namespace acb
