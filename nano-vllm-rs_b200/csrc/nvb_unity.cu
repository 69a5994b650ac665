// Single translation unit for libnvb.so (see internal.cuh).
#include "api.cu"
#include "decode.cu"
#include "decode_mma.cu"
#include "prefill.cu"
#include "qkv_rope.cu"
#include "static_scratch.cu"
#include "gather.cu"
#include "generic.cu"
