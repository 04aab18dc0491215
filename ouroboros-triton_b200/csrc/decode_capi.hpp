// Decode argument checks and split-K planning shared by the decode entry points.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "attention.hpp"
#include "ouroboros_b200.h"

namespace ouro::capi {

// Validated kernel parameters from the C struct (no split plan yet); throws CapiError.
DecodeParams decode_params(const ouro_decode_args* a);
// Kernel choice, blocks per split-K chunk, chunks per sequence, workspace bytes.
void decode_plan(DecodeParams& p, const ouro_decode_args* a, bool* use_tc, size_t* ws_bytes);
// Throws CapiError(OURO_ECUDA) carrying the CUDA error text.
void cuda_check(cudaError_t e, const char* what);
// Launches a planned decode (and its merge) with `workspace` of the planned size.
void decode_launch(DecodeParams& p, int dtype, bool tc, float* workspace, cudaStream_t st);

}  // namespace ouro::capi
