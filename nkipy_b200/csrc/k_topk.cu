// Top-k along the last axis (the reference's `topk` op: `core/ops/nn.py:65-152`,
// HLO TopK with largest = true; `is_ascend` is traced as negate -> topk -> negate).
//
// Output per row: the k largest values in descending order and their column
// indices (uint32).  Ties keep the lower index first.  The order is total and
// bit-exact: each element becomes a 64-bit key
//     (order-preserving 32-bit image of the value) << 32 | ~column
// so the largest key is the largest value at the smallest column.  Floats map
// by sign-magnitude flip (NaN sorts by its bit pattern: +NaN above +inf).
//
// One CTA per row (grid-stride over rows).  Round r finds the largest key
// strictly below the key of round r-1: k passes over the row, which sits in
// shared memory as 32-bit value images when it fits (cols <= 48K), else is
// re-read from global memory (L2).  Sized for sampling (k small, rows of a
// vocabulary shard).  The value written is the input element itself.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace nkb {
namespace topk {

constexpr int kThreads = 512;
constexpr int64_t kSmemCols = 48 * 1024;

__device__ __forceinline__ uint32_t order_bits(uint32_t bits, int dt) {
  switch (dt) {
    case NKB_F32: case NKB_BF16: case NKB_F16:  // widened to fp32 bits by load_as_reg
      return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    case NKB_I32: case NKB_I16: case NKB_I8: return bits ^ 0x80000000u;  // sign-extended by load_as_reg
    default: return bits;                                                 // unsigned, bool
  }
}

__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }

__device__ __forceinline__ uint64_t warp_max64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = umax64(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(kThreads) topk_rows_kernel(const void *__restrict__ x, int dt,
                                                             void *__restrict__ vals,
                                                             uint32_t *__restrict__ idx, int64_t rows,
                                                             int64_t cols, int k, int esize, bool staged) {
  extern __shared__ uint32_t s_img[];  // cols value images when staged
  __shared__ uint64_t s_warp[kThreads / 32];
  __shared__ uint64_t s_best;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * cols;
    if (staged) {
      for (int64_t c = tid; c < cols; c += kThreads) s_img[c] = order_bits(load_as_reg(x, base + c, dt), dt);
      __syncthreads();
    }
    uint64_t prev = ~0ull;
    bool first = true;
    for (int r = 0; r < k; ++r) {
      uint64_t best = 0;
      bool any = false;
      for (int64_t c = tid; c < cols; c += kThreads) {
        const uint32_t img = staged ? s_img[c] : order_bits(load_as_reg(x, base + c, dt), dt);
        const uint64_t key = ((uint64_t)img << 32) | (uint32_t)~(uint32_t)c;
        if (first || key < prev) {
          best = any ? umax64(best, key) : key;
          any = true;
        }
      }
      best = warp_max64(best);  // 0 is the smallest key and never wins over a real one
      if (lane == 0) s_warp[warp] = best;
      __syncthreads();
      if (warp == 0) {
        uint64_t v = lane < kThreads / 32 ? s_warp[lane] : 0;
        v = warp_max64(v);
        if (lane == 0) s_best = v;
      }
      __syncthreads();
      prev = s_best;
      first = false;
      if (tid == 0) {
        const uint32_t col = ~(uint32_t)(prev & 0xffffffffu);
        idx[row * k + r] = col;
        const uint8_t *src = static_cast<const uint8_t *>(x) + (base + col) * esize;
        uint8_t *dst = static_cast<uint8_t *>(vals) + (row * k + r) * esize;
        for (int b = 0; b < esize; ++b) dst[b] = src[b];
      }
      __syncthreads();  // s_best / s_warp are rewritten next round
    }
  }
}

int topk_any(const void *x, int dt, void *vals, uint32_t *idx, int64_t rows, int64_t cols, int64_t k,
             cudaStream_t stream, int device) {
  const int es = dtype_size(dt);
  if (!es || dt == NKB_F8E4M3 || dt == NKB_F8E5M2) return fail(NKB_ERR_UNSUPPORTED, "topk: dtype");
  if (k < 1 || k > cols) return fail(NKB_ERR_INVALID, "topk: k must be in [1, cols]");
  if (cols > 0xffffffffll) return fail(NKB_ERR_UNSUPPORTED, "topk: rows longer than 2^32");
  if (rows == 0) return NKB_OK;
  const bool staged = cols <= kSmemCols;
  const size_t smem = staged ? (size_t)cols * 4 : 0;
  if (smem > 48 * 1024)
    NKB_CUDA_TRY(cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t cap = (int64_t)num_sms(device) * (staged && smem > 64 * 1024 ? 1 : 2);
  topk_rows_kernel<<<(unsigned)std::min<int64_t>(rows, cap), kThreads, smem, stream>>>(x, dt, vals, idx, rows, cols,
                                                                                        (int)k, es, staged);
  return launch_status("topk_rows_kernel");
}

// "topk_rows": ptrs x values indices; ints rows cols k dtype
int check(const Step &s) {
  if (s.buf_ids.size() != 3 || s.ints.size() != 4) return fail(NKB_ERR_PLAN, "topk_rows: bad parameters");
  if (s.ints[2] < 1 || s.ints[2] > s.ints[1]) return fail(NKB_ERR_PLAN, "topk_rows: k out of range");
  return NKB_OK;
}
int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  return topk_any(a.ptrs[0], (int)q[3], a.ptrs[1], static_cast<uint32_t *>(a.ptrs[2]), q[0], q[1], q[2], a.stream,
                  a.device);
}

}  // namespace topk

NKB_REGISTER_KERNEL("topk_rows", topk::launch, topk::check);

}  // namespace nkb

extern "C" int nkb_topk_rows(const void *x, int dtype, void *values, uint32_t *indices, int64_t rows, int64_t cols,
                             int64_t k, void *stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  return nkb::topk::topk_any(x, dtype, values, indices, rows, cols, k, static_cast<cudaStream_t>(stream), dev);
}
