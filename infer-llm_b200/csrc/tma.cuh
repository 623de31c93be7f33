// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library needs no -lcuda) and the tiled-load helpers
// shared by the tcgen05 GEMM and the decode attention.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace b200 {

// F32 tensor of `rank` dims (dims[0] innermost, strides in bytes for dims 1..rank-1),
// boxes of box[0..rank). False if the driver entry point is missing or the encoding
// is rejected (alignment of base / strides, box limits).
bool tma_encode_f32(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides_bytes,
                    const uint32_t *box, CUtensorMapSwizzle swizzle);

B200_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z, uint32_t bar,
                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
        : "memory");
}

}  // namespace b200
