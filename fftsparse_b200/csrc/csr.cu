// csr.cu -- the selected blocks as a CSR index list (row_ptr, col_idx).
//
// The reference hands its attention kernel the bool block mask
// (base_blockmask, attn_src/fft_attn/my_attn_v7.py:780); a caller that wants
// the list of selected key blocks per query block (a block-sparse kernel taking
// indices, or an analysis of the selection) gets it here from the packed bits,
// without expanding the N x N mask:
//
//   row_ptr_kernel  one CTA: exclusive scan of the per-row block counts into
//                   int64 row_ptr[rows + 1] (row_ptr[rows] = number of kept blocks)
//   col_idx_kernel  one warp per row: each lane takes 32-bit words of the row,
//                   the warp's prefix sum of their popcounts places each lane's
//                   blocks, written in ascending block order
// rows = B * H * N in the bits' [B, H, N, W] order.  The fill checks every row's
// popcount against its row_ptr span and its end against col_idx's capacity; a
// row that fails is not written and the status word is set to 1.

#include "ffts_common.cuh"

namespace ffts {
namespace csr {

constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads) row_ptr_kernel(const int32_t *__restrict__ count, int64_t rows,
                                                                int64_t *__restrict__ row_ptr) {
  __shared__ int64_t warp_tot[kScanThreads / 32];
  __shared__ int64_t carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < rows; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const int64_t c = i < rows ? int64_t(count[i]) : 0;
    int64_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int64_t w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += t;
      }
      warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int64_t before = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + incl - c;
    if (i < rows) row_ptr[i] = before;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_tot[kScanThreads / 32 - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) row_ptr[rows] = carry;
}

__global__ void __launch_bounds__(256) col_idx_kernel(const uint32_t *__restrict__ bits, int64_t rows, int N, int W,
                                                       const int64_t *__restrict__ row_ptr,
                                                       int32_t *__restrict__ col_idx, int64_t capacity,
                                                       int32_t *__restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint32_t *r = bits + row * W;
  const int64_t start = row_ptr[row], end = row_ptr[row + 1];
  // popcount of the whole row (bits past N are ignored)
  int total = 0;
  for (int w = lane; w < W; w += 32) {
    uint32_t word = r[w];
    const int rem = N - w * 32;
    if (rem < 32) word &= (1u << rem) - 1u;
    total += __popc(word);
  }
  for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  if (int64_t(total) != end - start || end > capacity || start < 0) {
    if (lane == 0) atomicExch(status, 1);
    return;
  }
  int64_t base = start;
  for (int w0 = 0; w0 < W; w0 += 32) {
    const int w = w0 + lane;
    uint32_t word = w < W ? r[w] : 0u;
    const int rem = N - w * 32;
    if (w < W && rem < 32) word &= (1u << rem) - 1u;
    const int c = __popc(word);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int64_t pos = base + incl - c;
    while (word) {
      const int t = __ffs(word) - 1;
      word &= word - 1u;
      if (FFTS_IN_RANGE(pos, capacity)) col_idx[pos] = w * 32 + t;
      ++pos;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
}

}  // namespace csr

int mask_row_ptr(const int32_t *row_count, int64_t rows, int64_t *row_ptr, cudaStream_t stream) {
  FFTS_REQUIRE(row_count && row_ptr && rows >= 1, "mask_row_ptr: NULL argument or no rows");
  csr::row_ptr_kernel<<<1, csr::kScanThreads, 0, stream>>>(row_count, rows, row_ptr);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

int mask_col_idx(const uint32_t *bits, int64_t rows, int64_t N, const int64_t *row_ptr, int32_t *col_idx,
                 int64_t capacity, int32_t *status, cudaStream_t stream) {
  FFTS_REQUIRE(bits && row_ptr && status && rows >= 1 && N >= 1 && capacity >= 0 && (col_idx || capacity == 0),
               "mask_col_idx: bad argument");
  FFTS_REQUIRE(N <= kMaxBlocks, "mask_col_idx: N = %lld exceeds %d blocks", (long long)N, kMaxBlocks);
  const int64_t blocks = ceil_div(rows, int64_t(8));
  FFTS_REQUIRE(blocks < (int64_t(1) << 31), "mask_col_idx: too many rows");
  csr::col_idx_kernel<<<unsigned(blocks), 256, 0, stream>>>(bits, rows, int(N), int(ceil_div(N, int64_t(32))),
                                                            row_ptr, col_idx, capacity, status);
  FFTS_CUDA(cudaGetLastError());
  return FFTS_OK;
}

}  // namespace ffts
