// Paged-attention kernels for K/V half, query in another dtype (low-half residual MMA).
#include "attention_kernels.cuh"

namespace kvpd {
KVPD_DEFINE_VARIANT(f16_qres, __half, true)
}  // namespace kvpd
