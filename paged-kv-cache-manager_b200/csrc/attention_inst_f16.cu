// Paged-attention kernels for K/V half, query in the K/V dtype.
#include "attention_kernels.cuh"

namespace kvpd {
KVPD_DEFINE_VARIANT(f16, __half, false)
}  // namespace kvpd
