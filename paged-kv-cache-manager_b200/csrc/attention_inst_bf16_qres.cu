// Paged-attention kernels for K/V nv_bfloat16, query in another dtype (low-half residual MMA).
#include "attention_kernels.cuh"

namespace kvpd {
KVPD_DEFINE_VARIANT(bf16_qres, __nv_bfloat16, true)
}  // namespace kvpd
