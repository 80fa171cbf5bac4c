// Shapes and ops the tensor-core path does not cover yet report "unsupported"; the API
// layer then routes them to the SIMT kernels.
#include "pf_common.cuh"
#include "pf_tc.h"
namespace pf { namespace tc {
bool layernorm_supported(int, const void*, const void*) { return false; }
int layernorm_bf16(const void*, void*, const float*, const float*, int64_t, int, float, cudaStream_t) { return PF_EUNSUPPORTED; }
bool transition_supported(int, int) { return false; }
int transition(const pf_transition_params*, const void*, int64_t, void*, int64_t, int64_t, int, int, int, cudaStream_t) { return PF_EUNSUPPORTED; }
}}
