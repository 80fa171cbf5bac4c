// Temporary: tensor-core path not yet wired; every query reports "unsupported".
#include "pf_common.cuh"
#include "pf_tc.h"
namespace pf { namespace tc {
bool layernorm_supported(int, const void*, const void*) { return false; }
int layernorm_bf16(const void*, void*, const float*, const float*, int64_t, int, float, cudaStream_t) { return PF_EUNSUPPORTED; }
bool triatt_bias_supported(int, int) { return false; }
int triatt_bias(const pf_triatt_params*, pf_pair_view, int64_t, int64_t, void*, int64_t, int64_t, int, int, cudaStream_t) { return PF_EUNSUPPORTED; }
bool triatt_supported(int, int, int) { return false; }
size_t triatt_ws_bytes(int64_t, int64_t, int64_t, int, int, int) { return 0; }
int triatt(const pf_triatt_params*, pf_pair_view, pf_mask_view, const void*, int64_t, int64_t, pf_pair_view, int64_t, int64_t, int64_t, int64_t, int64_t, int, int, int, float, int, void*, size_t, cudaStream_t) { return PF_EUNSUPPORTED; }
bool transition_supported(int, int) { return false; }
int transition(const pf_transition_params*, const void*, int64_t, void*, int64_t, int64_t, int, int, int, cudaStream_t) { return PF_EUNSUPPORTED; }
}}
