// synth.cuh -- on-device synthetic weight generation (synth.cu).
#pragma once
#include "common.cuh"

namespace qma {

enum { KIND_W = 0, KIND_NORM, KIND_CONV, KIND_DT, KIND_A };

uint64_t name_key(const char *name, uint64_t seed);
int tensor_kind(const char *name);
// Generate `nelem` elements of tensor `name` in GGUF block order into dst.
int synth_tensor_gguf(const char *name, int type, uint64_t nelem, uint64_t seed, void *dst,
                      cudaStream_t st);

}  // namespace qma
