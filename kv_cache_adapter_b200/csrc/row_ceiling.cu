// Roofline reference for moves of randomly placed rows (kvca_row_ceiling).
//
// The copy bandwidth of the GPU is the ceiling of sequential moves; a move
// whose rows sit at random places in HBM has a lower one, set by the DRAM
// access pattern (short random bursts open more DRAM rows per byte).  This
// kernel moves rows through a 32-bit permutation with no other index work:
// one plane, no block / slot arithmetic, no chunk layout, the permutation
// read once per row.  Each row goes to a group of lanes (a lane per 16-byte
// vector up to 32 lanes; 576-byte rows, 36 vectors, take 4 lanes of 9), and
// each lane group keeps 2 or 4 rows in flight.  What it reaches for a
// row width is the measured ceiling the movers' random-row fractions are
// judged against.  It is a measurement aid, not part of any adapter path.

#include <cuda_runtime.h>
#include <stdint.h>

#include "kvca.h"

namespace {

constexpr int kCeilThreads = 256;

template <int kVpr, bool kScatter>
__global__ void __launch_bounds__(kCeilThreads) row_ceiling_kernel(const uint4* __restrict__ src,
                                                                   uint4* __restrict__ dst,
                                                                   const uint32_t* __restrict__ perm,
                                                                   uint32_t rows) {
  constexpr int kLanes = kVpr % 32 == 0 ? 32 : (kVpr % 16 == 0 ? 16 : (kVpr % 8 == 0 ? 8 : (kVpr % 4 == 0 ? 4 : 1)));
  constexpr int kVpl = kVpr / kLanes;
  static_assert(kVpl * kLanes == kVpr, "lanes must tile the row");
  constexpr int kCeilRows = kVpl >= 8 ? 2 : 4;  // rows in flight per lane group
  const uint32_t gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t groups = gridDim.x * blockDim.x / kLanes;
  const uint32_t g = gtid / kLanes;
  const uint32_t l = gtid % kLanes;
  for (uint32_t r0 = g * kCeilRows; r0 < rows; r0 += groups * kCeilRows) {
    uint4 buf[kCeilRows][kVpl];
    uint32_t pr[kCeilRows];
#pragma unroll
    for (int u = 0; u < kCeilRows; ++u) pr[u] = r0 + u < rows ? perm[r0 + u] : rows;
#pragma unroll
    for (int u = 0; u < kCeilRows; ++u) {
      if (pr[u] < rows) {  // out-of-range permutation entries are skipped
        const size_t s = static_cast<size_t>(kScatter ? r0 + u : pr[u]) * kVpr + l;
#pragma unroll
        for (int v = 0; v < kVpl; ++v) buf[u][v] = __ldcs(src + s + v * kLanes);
      }
    }
#pragma unroll
    for (int u = 0; u < kCeilRows; ++u) {
      if (pr[u] < rows) {
        const size_t d = static_cast<size_t>(kScatter ? pr[u] : r0 + u) * kVpr + l;
#pragma unroll
        for (int v = 0; v < kVpl; ++v) __stcs(dst + d + v * kLanes, buf[u][v]);
      }
    }
  }
}

template <int kVpr>
cudaError_t launch_ceiling(const void* src, void* dst, const uint32_t* perm, uint32_t rows, bool scatter, int ctas,
                           cudaStream_t stream) {
  if (scatter)
    row_ceiling_kernel<kVpr, true><<<ctas, kCeilThreads, 0, stream>>>(static_cast<const uint4*>(src),
                                                                      static_cast<uint4*>(dst), perm, rows);
  else
    row_ceiling_kernel<kVpr, false><<<ctas, kCeilThreads, 0, stream>>>(static_cast<const uint4*>(src),
                                                                       static_cast<uint4*>(dst), perm, rows);
  return cudaGetLastError();
}

}  // namespace

extern "C" int kvca_row_ceiling(const void* d_src, void* d_dst, const uint32_t* d_perm, int64_t rows,
                                int64_t row_bytes, int scatter, int ctas, kvca_stream_t stream) {
  if (d_src == nullptr || d_dst == nullptr || d_perm == nullptr || rows < 1 || rows >= (int64_t{1} << 31) ||
      ctas < 1 || (reinterpret_cast<uintptr_t>(d_src) | reinterpret_cast<uintptr_t>(d_dst)) % 16 != 0)
    return KVCA_ERR_BAD_ARGUMENT;
  const uint32_t n = static_cast<uint32_t>(rows);
  const bool s = scatter != 0;
  cudaError_t e;
  switch (row_bytes) {
    case 64: e = launch_ceiling<4>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    case 128: e = launch_ceiling<8>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    case 256: e = launch_ceiling<16>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    case 576: e = launch_ceiling<36>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    case 1152: e = launch_ceiling<72>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    case 2048: e = launch_ceiling<128>(d_src, d_dst, d_perm, n, s, ctas, stream); break;
    default: return KVCA_ERR_BAD_ARGUMENT;
  }
  return e == cudaSuccess ? KVCA_OK : KVCA_ERR_CUDA;
}
