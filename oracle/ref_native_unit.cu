// Build unit for the reference's own native kernels, compiled from the
// sources where they lie (see oracle/Makefile). TEST INFRASTRUCTURE ONLY:
// it produces oracle/_ref/libref_native.so, the second oracle (the
// reference's nv_attention, nv_qkv_rope_cached, nv_rope_cache and the
// split-KV decode candidate) that GPU parity tests compare against.
// decode_candidate.cuh documents that it is included after kernels.cu.
#include "kernels.cu"
#include "decode_candidate.cuh"
