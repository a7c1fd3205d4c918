// Paged-attention kernels for K/V nv_bfloat16, query in the K/V dtype.
#include "attention_kernels.cuh"

namespace kvpd {
KVPD_DEFINE_VARIANT(bf16, __nv_bfloat16, false)
}  // namespace kvpd
