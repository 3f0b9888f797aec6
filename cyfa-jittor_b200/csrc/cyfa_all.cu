// Single translation unit of the CyFA CUDA library (libcyfa.so): every kernel
// file and the C-ABI are compiled together so that device globals (the error
// word) and templates need no relocatable device code.
#include "cyfa_common.cuh"
#include "selftest.cu"
#include "decode.cu"
#include "prep.cu"
#include "gla_fwd.cu"
#include "gla_bwd.cu"
#include "layer.cu"
#include "capi.cu"
#include "chunk_api.cu"
#include "layer_api.cu"
#include "gate_norm.cu"
#include "noalloc.cu"
#include "lm_decode.cu"
#include "gradbuf.cu"
