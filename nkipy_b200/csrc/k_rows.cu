// Row kernels: last-axis softmax, residual-add + RMSNorm, first-occurrence
// argmax, and a generic strided reduction.
//
// softmax_rows / rmsnorm_rows keep a whole row in registers (one HBM read,
// one HBM write per element): the row is split over THREADS threads in
// 4-element chunks loaded with 16-byte (fp32) or 8-byte (bf16) vector loads,
// reductions use warp shuffles and, across warps, a small shared-memory
// array.  Short rows use one warp per row so that a CTA still moves enough
// bytes; rows longer than the register budget stream twice through L2.
//
// Numerics follow the traced NumPy compositions (reference
// tests/kernels/softmax.py:7-10; qwen3_embedding/kernels/rmsnorm.py:4-16):
// fp32 accumulation, exp(x - max) / sum with IEEE division, and
// h / sqrt(sum(h*h)/N + eps) * w in that order.

#include <float.h>
#include <math.h>

#include "common.cuh"

namespace nkb {
namespace rows {

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  using type = float4;
};
template <>
struct Vec4<__nv_bfloat16> {
  using type = uint2;  // 4 x bf16
};

__device__ __forceinline__ void load4(const float *p, float *v) {
  float4 t = *reinterpret_cast<const float4 *>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16 *p, float *v) {
  uint2 t = *reinterpret_cast<const uint2 *>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&t.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&t.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
__device__ __forceinline__ void store4(float *p, const float *v) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16 *p, const float *v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t *>(&a);
  t.y = *reinterpret_cast<uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(p) = t;
}
__device__ __forceinline__ float load1(const float *p) { return *p; }
__device__ __forceinline__ float load1(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load1(const __half *p) { return __half2float(*p); }
__device__ __forceinline__ void store1(float *p, float v) { *p = v; }
__device__ __forceinline__ void store1(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

template <int THREADS>
__device__ __forceinline__ float row_reduce_max(float v, float *smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (THREADS > 32) {
    const int w = threadIdx.x / 32, l = threadIdx.x % 32;
    __syncthreads();
    if (l == 0) smem[w] = v;
    __syncthreads();
    v = (l < THREADS / 32) ? smem[l] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  }
  return v;
}

template <int THREADS>
__device__ __forceinline__ float row_reduce_sum(float v, float *smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (THREADS > 32) {
    const int w = threadIdx.x / 32, l = threadIdx.x % 32;
    __syncthreads();
    if (l == 0) smem[w] = v;
    __syncthreads();
    v = (l < THREADS / 32) ? smem[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  return v;
}

// ---------------------------------------------------------------------------
// softmax
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row softmax held in registers: THREADS threads per row (32 or 256), CHUNKS
// 4-element chunks per thread, 256 / THREADS rows per CTA.  Persistent: a grid
// of MINB CTAs per SM walks the rows, and the loads of a thread's next row are
// issued before the current row is reduced, so about MINB x 256 x CHUNKS x 16
// bytes per SM stay in flight from HBM across the reductions.  exp is
// ex2.approx of (x - max)·log2(e) and the division a multiply by the rounded
// reciprocal of the sum: within a few ulp of exp(x - max) / sum, far inside
// the fp32 tolerance of the path.  cols must be a multiple of 4 here.
template <int CHUNKS>
constexpr int softmax_minb() {
  return CHUNKS <= 1 ? 8 : CHUNKS <= 2 ? 6 : CHUNKS <= 4 ? 5 : 2;
}

template <int THREADS, int CHUNKS, typename Tin, typename Tout>
__global__ void __launch_bounds__(256, softmax_minb<CHUNKS>())
    softmax_reg_kernel(const Tin *__restrict__ x, Tout *__restrict__ y, int64_t rows, int cols) {
  // [0]: per-warp maxima, [1]: per-warp sums (256-thread rows only); one
  // buffer each, so a row needs two CTA barriers
  __shared__ float red[2][8];
  constexpr int RPB = 256 / THREADS;
  constexpr float LOG2E = 1.4426950408889634f;
  const int sub = threadIdx.x / THREADS;
  const int t = threadIdx.x % THREADS;
  const int64_t stride = (int64_t)gridDim.x * RPB;
  float nx[CHUNKS][4];
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * THREADS + t) * 4;
      if (r < rows && col < cols) {
        load4(x + r * cols + col, nx[c]);
      } else {
        nx[c][0] = nx[c][1] = nx[c][2] = nx[c][3] = -INFINITY;
      }
    }
  };
  int64_t row = (int64_t)blockIdx.x * RPB + sub;
  fetch(row);
  // 256-thread rows: the CTA walks rows together (row is CTA-uniform)
  for (; row < rows; row += stride) {
    float v[CHUNKS][4];
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) v[c][j] = nx[c][j];
    fetch(row + stride);
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, v[c][j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (THREADS > 32) {
      if (t % 32 == 0) red[0][t / 32] = m;
      __syncthreads();
      m = red[0][t % 8];
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[c][j] = ex2_approx((v[c][j] - m) * LOG2E);
        s += v[c][j];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (THREADS > 32) {
      if (t % 32 == 0) red[1][t / 32] = s;
      __syncthreads();
      s = red[1][t % 8];
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    const float inv = __frcp_rn(s);
    Tout *yr = y + row * cols;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * THREADS + t) * 4;
      if (col < cols) {
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = v[c][j] * inv;
        store4(yr + col, o);
      }
    }
  }
}

template <int THREADS, int CHUNKS, typename Tin, typename Tout>
int softmax_reg_launch(const Tin *x, Tout *y, int64_t rows, int cols, cudaStream_t st, int device) {
  constexpr int RPB = 256 / THREADS;
  const unsigned grid = (unsigned)std::min<int64_t>((rows + RPB - 1) / RPB,
                                                    (int64_t)num_sms(device) * softmax_minb<CHUNKS>());
  softmax_reg_kernel<THREADS, CHUNKS, Tin, Tout><<<grid, 256, 0, st>>>(x, y, rows, cols);
  return launch_status("softmax_rows");
}

// Rows too long for registers (or cols % 4 != 0): online max/sum pass, then
// a second pass that re-reads the row (from L2 for moderate rows).
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) softmax_stream_kernel(const Tin *__restrict__ x, Tout *__restrict__ y,
                                                             int64_t rows, int64_t cols) {
  __shared__ float smem[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const Tin *xr = x + row * cols;
    float m = -INFINITY, s = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float v = load1(xr + c);
      if (v > m) {
        s = s * expf(m - v) + 1.f;
        m = v;
      } else {
        s += expf(v - m);
      }
    }
    const float gm = row_reduce_max<256>(m, smem);
    s = (m == -INFINITY) ? 0.f : s * expf(m - gm);
    s = row_reduce_sum<256>(s, smem);
    Tout *yr = y + row * cols;
    for (int64_t c = threadIdx.x; c < cols; c += 256) store1(yr + c, __fdiv_rn(expf(load1(xr + c) - gm), s));
    __syncthreads();
  }
}

template <typename Tin, typename Tout>
int softmax_dispatch(const void *x, void *y, int64_t rows, int64_t cols, cudaStream_t st, int device) {
  if (rows == 0 || cols == 0) return NKB_OK;
  const Tin *xi = static_cast<const Tin *>(x);
  Tout *yo = static_cast<Tout *>(y);
  const bool aligned = (cols % 4 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0);
  const int64_t cap = (int64_t)num_sms(device) * 32;
  auto grid = [&](int rpb) { return (unsigned)std::min<int64_t>((rows + rpb - 1) / rpb, cap); };
  if (aligned && cols <= 1024) {
    const int chunks = (int)((cols + 127) / 128);
    if (chunks <= 1) return softmax_reg_launch<32, 1>(xi, yo, rows, (int)cols, st, device);
    if (chunks <= 2) return softmax_reg_launch<32, 2>(xi, yo, rows, (int)cols, st, device);
    if (chunks <= 4) return softmax_reg_launch<32, 4>(xi, yo, rows, (int)cols, st, device);
    return softmax_reg_launch<32, 8>(xi, yo, rows, (int)cols, st, device);
  } else if (aligned && cols <= 8192) {
    const int chunks = (int)((cols + 1023) / 1024);
    if (chunks <= 1) return softmax_reg_launch<256, 1>(xi, yo, rows, (int)cols, st, device);
    if (chunks <= 2) return softmax_reg_launch<256, 2>(xi, yo, rows, (int)cols, st, device);
    if (chunks <= 4) return softmax_reg_launch<256, 4>(xi, yo, rows, (int)cols, st, device);
    return softmax_reg_launch<256, 8>(xi, yo, rows, (int)cols, st, device);
  } else {
    softmax_stream_kernel<Tin, Tout><<<grid(1), 256, 0, st>>>(xi, yo, rows, cols);
  }
  return launch_status("softmax_rows");
}

int softmax_any(const void *x, int xdt, void *y, int ydt, int64_t rows, int64_t cols, cudaStream_t st, int dev) {
  if (xdt == NKB_F32 && ydt == NKB_F32) return softmax_dispatch<float, float>(x, y, rows, cols, st, dev);
  if (xdt == NKB_BF16 && ydt == NKB_BF16)
    return softmax_dispatch<__nv_bfloat16, __nv_bfloat16>(x, y, rows, cols, st, dev);
  if (xdt == NKB_BF16 && ydt == NKB_F32) return softmax_dispatch<__nv_bfloat16, float>(x, y, rows, cols, st, dev);
  if (xdt == NKB_F32 && ydt == NKB_BF16) return softmax_dispatch<float, __nv_bfloat16>(x, y, rows, cols, st, dev);
  return fail(NKB_ERR_UNSUPPORTED, "softmax_rows: dtype combination not supported");
}

// ---------------------------------------------------------------------------
// residual add + RMSNorm
// ---------------------------------------------------------------------------
template <int THREADS, int CHUNKS, typename T, typename TW, bool RES, bool SUM_OUT>
__global__ void __launch_bounds__(256) rmsnorm_reg_kernel(const T *__restrict__ x, const T *__restrict__ r,
                                                          const TW *__restrict__ w, T *__restrict__ y,
                                                          T *__restrict__ hsum, int64_t rows, int cols, float eps,
                                                          int64_t xin, int64_t xos) {
  __shared__ float smem[32];
  constexpr int RPB = 256 / THREADS;
  const int sub = threadIdx.x / THREADS;
  const int t = threadIdx.x % THREADS;
  const float inv_n = (float)cols;
  for (int64_t row = (int64_t)blockIdx.x * RPB + sub; row - sub < rows; row += (int64_t)gridDim.x * RPB) {
    const bool active = row < rows;
    const int64_t arow = active ? row : 0;
    const int64_t base = arow * cols;
    const int64_t ibase = (arow / xin) * xos + (arow % xin) * cols;  // input rows: blocks of xin rows
    float v[CHUNKS][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * THREADS + t) * 4;
      if (active && col < cols) {
        load4(x + ibase + col, v[c]);
        if (RES) {
          float rv[4];
          load4(r + ibase + col, rv);
#pragma unroll
          for (int j = 0; j < 4; ++j) v[c][j] += rv[j];
          if (sizeof(T) == 2) {
            // the residual sum is a bf16 tensor in the trace: round it first
#pragma unroll
            for (int j = 0; j < 4; ++j) v[c][j] = __bfloat162float(__float2bfloat16_rn(v[c][j]));
          }
        }
      } else {
        v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += v[c][j] * v[c][j];
    }
    ss = row_reduce_sum<THREADS>(ss, smem);
    const float denom = sqrtf(__fdiv_rn(ss, inv_n) + eps);
    if (active) {
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * THREADS + t) * 4;
        if (col < cols) {
          if (SUM_OUT) store4(hsum + base + col, v[c]);
          float wv[4], o[4];
          load4(w + col, wv);
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = __fdiv_rn(v[c][j], denom) * wv[j];
          store4(y + base + col, o);
        }
      }
    }
  }
}

template <typename T, typename TW, bool RES, bool SUM_OUT>
__global__ void __launch_bounds__(256) rmsnorm_stream_kernel(const T *__restrict__ x, const T *__restrict__ r,
                                                             const TW *__restrict__ w, T *__restrict__ y,
                                                             T *__restrict__ hsum, int64_t rows, int64_t cols,
                                                             float eps, int64_t xin, int64_t xos) {
  __shared__ float smem[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * cols;
    const int64_t ibase = (row / xin) * xos + (row % xin) * cols;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      float h = load1(x + ibase + c);
      if (RES) {
        h += load1(r + ibase + c);
        if (sizeof(T) == 2) h = __bfloat162float(__float2bfloat16_rn(h));
      }
      ss += h * h;
    }
    ss = row_reduce_sum<256>(ss, smem);
    const float denom = sqrtf(__fdiv_rn(ss, (float)cols) + eps);
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      float h = load1(x + ibase + c);
      if (RES) {
        h += load1(r + ibase + c);
        if (sizeof(T) == 2) h = __bfloat162float(__float2bfloat16_rn(h));
      }
      if (SUM_OUT) store1(hsum + base + c, h);
      store1(y + base + c, __fdiv_rn(h, denom) * load1(w + c));
    }
    __syncthreads();
  }
}

// bf16 rows of up to 8192 columns (the decoder layer's norms): 256 threads, 8
// consecutive columns per thread per chunk (16-byte loads and stores), the row
// sum rounded to bf16 as the trace does, and the normalisation as a multiply
// by the reciprocal of sqrt(mean + eps) (within one fp32 ulp of the division,
// the result then rounded to bf16).
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float *v) {
  const uint4 t = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float *p, float *v) {
  const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float *v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t *>(&h);
  }
  *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int CHUNKS, typename TW, bool RES, bool SUM_OUT>
__global__ void __launch_bounds__(256) rmsnorm_bf16_kernel(const __nv_bfloat16 *__restrict__ x,
                                                           const __nv_bfloat16 *__restrict__ r,
                                                           const TW *__restrict__ w, __nv_bfloat16 *__restrict__ y,
                                                           __nv_bfloat16 *__restrict__ hsum, int64_t rows, int cols,
                                                           float eps, int64_t xin, int64_t xos) {
  __shared__ float smem[32];
  const int t = threadIdx.x;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * cols;
    const int64_t ibase = (row / xin) * xos + (row % xin) * cols;
    float v[CHUNKS][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * 256 + t) * 8;
      if (col < cols) {
        load8(x + ibase + col, v[c]);
        if (RES) {
          float rv[8];
          load8(r + ibase + col, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[c][j] = __bfloat162float(__float2bfloat16_rn(v[c][j] + rv[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
    }
    ss = row_reduce_sum<256>(ss, smem);
    const float inv = 1.0f / sqrtf(__fdiv_rn(ss, (float)cols) + eps);
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int col = (c * 256 + t) * 8;
      if (col < cols) {
        if (SUM_OUT) store8(hsum + base + col, v[c]);
        float wv[8], o[8];
        load8(w + col, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[c][j] * inv * wv[j];
        store8(y + base + col, o);
      }
    }
  }
}

// CTAs of `kernel` (256 threads, no dynamic shared memory) that fit on the
// device at once: a grid-stride kernel sized to this runs in one wave (a
// larger grid leaves a second, partial wave of whole CTAs at the end).
template <class K>
int64_t resident_ctas_256(K kernel, int device) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<const void *, int>, int>> cache;
  const void *key = reinterpret_cast<const void *>(kernel);
  std::lock_guard<std::mutex> lk(mu);
  for (auto &e : cache)
    if (e.first.first == key && e.first.second == device) return (int64_t)num_sms(device) * e.second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 256, 0) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 1;
  }
  cache.push_back({{key, device}, n});
  return (int64_t)num_sms(device) * n;
}

template <typename T, typename TW, bool RES, bool SUM_OUT>
int rmsnorm_dispatch3(const void *x, const void *r, const void *w, void *y, void *hs, int64_t rows, int64_t cols,
                      float eps, int64_t xin, int64_t xos, cudaStream_t st, int device) {
  const T *xi = static_cast<const T *>(x);
  const T *ri = static_cast<const T *>(r);
  const TW *wi = static_cast<const TW *>(w);
  T *yo = static_cast<T *>(y);
  T *ho = static_cast<T *>(hs);
  const bool aligned = (cols % 4 == 0) && (xos % 4 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) &&
                       ((uintptr_t)w % 16 == 0) && (!RES || (uintptr_t)r % 16 == 0) &&
                       (!SUM_OUT || (uintptr_t)hs % 16 == 0);
  const int64_t cap = (int64_t)num_sms(device) * 32;
  auto grid = [&](int rpb) { return (unsigned)std::min<int64_t>((rows + rpb - 1) / rpb, cap); };
  if constexpr (sizeof(T) == 2) {
    const bool a16 = aligned && cols % 8 == 0 && xos % 8 == 0 && cols > 1024 && cols <= 8192;
    if (a16) {
      auto go = [&](auto kern) {
        const unsigned g = (unsigned)std::min<int64_t>(rows, resident_ctas_256(kern, device));
        kern<<<g, 256, 0, st>>>(xi, ri, wi, yo, ho, rows, (int)cols, eps, xin, xos);
      };
      if (cols <= 2048)
        go(rmsnorm_bf16_kernel<1, TW, RES, SUM_OUT>);
      else if (cols <= 4096)
        go(rmsnorm_bf16_kernel<2, TW, RES, SUM_OUT>);
      else
        go(rmsnorm_bf16_kernel<4, TW, RES, SUM_OUT>);
      return launch_status("rmsnorm_rows");
    }
  }
#define RMS_LAUNCH(TH, CH, RPB) \
  rmsnorm_reg_kernel<TH, CH, T, TW, RES, SUM_OUT><<<grid(RPB), 256, 0, st>>>(xi, ri, wi, yo, ho, rows, (int)cols, eps, \
                                                                       xin, xos)
  if (aligned && cols <= 1024) {
    const int ch = (int)((cols + 127) / 128);
    if (ch <= 1) RMS_LAUNCH(32, 1, 8);
    else if (ch <= 2) RMS_LAUNCH(32, 2, 8);
    else if (ch <= 4) RMS_LAUNCH(32, 4, 8);
    else RMS_LAUNCH(32, 8, 8);
  } else if (aligned && cols <= 8192) {
    const int ch = (int)((cols + 1023) / 1024);
    if (ch <= 1) RMS_LAUNCH(256, 1, 1);
    else if (ch <= 2) RMS_LAUNCH(256, 2, 1);
    else if (ch <= 4) RMS_LAUNCH(256, 4, 1);
    else RMS_LAUNCH(256, 8, 1);
  } else {
    rmsnorm_stream_kernel<T, TW, RES, SUM_OUT><<<grid(1), 256, 0, st>>>(xi, ri, wi, yo, ho, rows, cols, eps, xin, xos);
  }
#undef RMS_LAUNCH
  return launch_status("rmsnorm_rows");
}

template <typename T, typename TW>
int rmsnorm_dispatch2(const void *x, const void *r, const void *w, void *y, void *hs, int64_t rows, int64_t cols,
                      float eps, int64_t xin, int64_t xos, cudaStream_t st, int dev) {
  if (r && hs) return rmsnorm_dispatch3<T, TW, true, true>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
  if (r) return rmsnorm_dispatch3<T, TW, true, false>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
  return rmsnorm_dispatch3<T, TW, false, false>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
}

// Input rows (x and the residual) come in blocks of ``xin`` consecutive rows,
// blocks ``xos`` elements apart (xin = rows: dense); output rows are dense.
int rmsnorm_any(const void *x, const void *r, const void *w, void *y, void *hs, int dt, int wdt, int64_t rows,
                int64_t cols, float eps, cudaStream_t st, int dev, int64_t xin, int64_t xos) {
  if (rows == 0 || cols == 0) return NKB_OK;
  if (!r && hs) return fail(NKB_ERR_INVALID, "rmsnorm_rows: sum output requires a residual input");
  if (xin <= 0 || rows % xin || xos < xin * cols) return fail(NKB_ERR_INVALID, "rmsnorm_rows: bad input row blocks");
  if (dt == NKB_F32 && wdt == NKB_F32)
    return rmsnorm_dispatch2<float, float>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
  if (dt == NKB_BF16 && wdt == NKB_BF16)
    return rmsnorm_dispatch2<__nv_bfloat16, __nv_bfloat16>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
  if (dt == NKB_BF16 && wdt == NKB_F32)
    return rmsnorm_dispatch2<__nv_bfloat16, float>(x, r, w, y, hs, rows, cols, eps, xin, xos, st, dev);
  return fail(NKB_ERR_UNSUPPORTED, "rmsnorm_rows: dtype combination not supported");
}

// ---------------------------------------------------------------------------
// RMSNorm of per-head rows followed by the half-split rotary embedding
// ---------------------------------------------------------------------------
// The q/k path of the Qwen3 attention (examples/models/qwen3/kernels/
// attention.py:103-118, rmsnorm.py:4-21, rope.py:34-57): every (token, head)
// row of head_dim = 2 * half bf16 values is normalised in fp32 and rounded to
// bf16, then rotated with the cos / sin row of its position, each traced bf16
// node rounded:  lo = r(r(x0 * cos) - r(x1 * sin)),  hi = r(r(x0 * sin) + r(x1 * cos)).
// One warp per row, lane l owning columns 4l..4l+3, its partner half one
// shuffle away.  Table row of row r: clamp(pos) (a run-time position, the
// traced gather) plus, for per-token tables, the token index (r / H) % S.
struct RopeRows {
  const __nv_bfloat16 *cos, *sin;
  int64_t tstride;    // elements between table rows
  const void *pos;    // nullable: position 0
  int pos_dt;
  int64_t T, S, H;    // table rows (clamp bound), tokens, heads
  int per_token;
};

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One launch may carry two row sets (the q and the k heads of a decode step):
// blocks [0, seg[0].blocks) take the first, the rest the second.
struct RopeSeg {
  const __nv_bfloat16 *x;
  const void *w;
  __nv_bfloat16 *y;
  int64_t rows, xin, xos;
  RopeRows rp;
  unsigned blocks;
};
struct RopeLaunch {
  RopeSeg seg[2];
  int nseg, cols;
  float eps;
};

template <typename TW>
__global__ void __launch_bounds__(256) rmsnorm_rope_kernel(const __grid_constant__ RopeLaunch L) {
  pdl_wait();
  pdl_trigger();
  const int si = (L.nseg > 1 && blockIdx.x >= L.seg[0].blocks) ? 1 : 0;
  const RopeSeg &S = L.seg[si];
  const __nv_bfloat16 *__restrict__ x = S.x;
  const TW *__restrict__ w = static_cast<const TW *>(S.w);
  __nv_bfloat16 *__restrict__ y = S.y;
  const int64_t rows = S.rows, xin = S.xin, xos = S.xos;
  const int cols = L.cols;
  const float eps = L.eps;
  const RopeRows &rp = S.rp;
  const int64_t bx = (int64_t)blockIdx.x - (si ? L.seg[0].blocks : 0);
  const int lane = threadIdx.x % 32;
  const int half = cols / 2;
  const int col = 4 * lane;
  const bool has = col < cols;
  int64_t p0 = 0;
  if (rp.pos) {
    const uint32_t raw = load_as_reg(rp.pos, 0, rp.pos_dt);
    p0 = (rp.pos_dt == NKB_U32 || rp.pos_dt == NKB_U16 || rp.pos_dt == NKB_U8) ? (int64_t)raw : (int64_t)(int32_t)raw;
    p0 = p0 < 0 ? 0 : (p0 >= rp.T ? rp.T - 1 : p0);
  }
  for (int64_t row = (bx * 256 + threadIdx.x) / 32; row < rows; row += (int64_t)S.blocks * 8) {
    const int64_t ibase = (row / xin) * xos + (row % xin) * cols;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (has) load4(x + ibase + col, v);
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float denom = sqrtf(__fdiv_rn(ss, (float)cols) + eps);
    float o[4];
    if (has) {
      float wv[4];
      load4(w + col, wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = bf16_round(__fdiv_rn(v[j], denom) * wv[j]);
    } else {
      o[0] = o[1] = o[2] = o[3] = 0.f;
    }
    float other[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) other[j] = __shfl_xor_sync(0xffffffffu, o[j], half / 4);
    if (has) {
      const bool lo = col < half;
      const int d = lo ? col : col - half;
      const int64_t t = p0 + (rp.per_token ? (row / rp.H) % rp.S : 0);
      float cs[4], sn[4];
      load4(rp.cos + t * rp.tstride + d, cs);
      load4(rp.sin + t * rp.tstride + d, sn);
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x0 = lo ? o[j] : other[j], x1 = lo ? other[j] : o[j];
        r[j] = lo ? bf16_round(bf16_round(x0 * cs[j]) - bf16_round(x1 * sn[j]))
                  : bf16_round(bf16_round(x0 * sn[j]) + bf16_round(x1 * cs[j]));
      }
      store4(y + row * cols + col, r);
    }
  }
}

// Validates one row set and fills its launch record (blocks: 8 rows each, at
// most 8 CTAs per SM).
static int rope_seg(const void *x, const void *w, void *y, int wdt, int64_t rows, int64_t cols, int64_t xin,
                    int64_t xos, const RopeRows &rp, int dev, RopeSeg *out) {
  if (cols != 64 && cols != 128) return fail(NKB_ERR_UNSUPPORTED, "rmsnorm_rope_rows: head_dim must be 64 or 128");
  if (xin <= 0 || rows % xin || xos < xin * cols || xos % 4)
    return fail(NKB_ERR_INVALID, "rmsnorm_rope_rows: bad input row blocks");
  if (rp.T < 1 || rp.S < 1 || rp.H < 1 || rp.tstride < cols / 2 || rp.tstride % 4)
    return fail(NKB_ERR_INVALID, "rmsnorm_rope_rows: bad table geometry");
  // 4 bf16 (8 bytes) per lane; an fp32 weight is read 16 bytes at a time
  if ((((uintptr_t)x | (uintptr_t)y | (uintptr_t)rp.cos | (uintptr_t)rp.sin) & 7) ||
      ((uintptr_t)w & (wdt == NKB_F32 ? 15 : 7)))
    return fail(NKB_ERR_UNSUPPORTED, "rmsnorm_rope_rows: operands not aligned for vector loads");
  if (wdt != NKB_BF16 && wdt != NKB_F32) return fail(NKB_ERR_UNSUPPORTED, "rmsnorm_rope_rows: weight dtype");
  out->x = static_cast<const __nv_bfloat16 *>(x);
  out->w = w;
  out->y = static_cast<__nv_bfloat16 *>(y);
  out->rows = rows;
  out->xin = xin;
  out->xos = xos;
  out->rp = rp;
  out->blocks = (unsigned)std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms(dev) * 8);
  return NKB_OK;
}

static int rope_launch(RopeLaunch &L, int wdt, cudaStream_t st, bool pdl) {
  unsigned grid = 0;
  for (int i = 0; i < L.nseg; ++i) grid += L.seg[i].blocks;
  if (grid == 0) return NKB_OK;
  if (wdt == NKB_BF16)
    launch_pdl(pdl, rmsnorm_rope_kernel<__nv_bfloat16>, grid, 256, 0, st, L);
  else
    launch_pdl(pdl, rmsnorm_rope_kernel<float>, grid, 256, 0, st, L);
  return launch_status("rmsnorm_rope_kernel");
}

// ---------------------------------------------------------------------------
// argmax / argmin over the last axis: first occurrence of the extreme value
// (reference core/ops/reduce.py:227-311 lowers it to max -> compare -> iota
// -> select -> min, i.e. the smallest index holding the maximum).
// ---------------------------------------------------------------------------
template <typename T, bool IS_MAX>
__global__ void __launch_bounds__(256) argext_kernel(const T *__restrict__ x, int32_t *__restrict__ out, int64_t rows,
                                                     int64_t cols) {
  __shared__ float sv[8];
  __shared__ int64_t si[8];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T *xr = x + row * cols;
    float best = IS_MAX ? -INFINITY : INFINITY;
    int64_t bi = cols;  // sentinel: larger than any index
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float v = load1(xr + c);
      if (IS_MAX ? (v > best) : (v < best)) {
        best = v;
        bi = c;
      } else if (v == best && c < bi) {
        bi = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if ((IS_MAX ? ov > best : ov < best) || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    const int w = threadIdx.x / 32, l = threadIdx.x % 32;
    if (l == 0) {
      sv[w] = best;
      si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int k = 1; k < 8; ++k)
        if ((IS_MAX ? sv[k] > best : sv[k] < best) || (sv[k] == best && si[k] < bi)) {
          best = sv[k];
          bi = si[k];
        }
      // all-NaN / empty rows: report 0 like an all-equal row
      out[row] = (int32_t)(bi >= cols ? 0 : bi);
    }
    __syncthreads();
  }
}

int argext_any(const void *x, int dt, int32_t *out, int64_t rows, int64_t cols, bool is_max, cudaStream_t st,
               int dev) {
  if (rows == 0) return NKB_OK;
  const unsigned g = (unsigned)std::min<int64_t>(rows, (int64_t)num_sms(dev) * 8);
  if (dt == NKB_F32) {
    if (is_max) argext_kernel<float, true><<<g, 256, 0, st>>>((const float *)x, out, rows, cols);
    else argext_kernel<float, false><<<g, 256, 0, st>>>((const float *)x, out, rows, cols);
  } else if (dt == NKB_BF16) {
    if (is_max) argext_kernel<__nv_bfloat16, true><<<g, 256, 0, st>>>((const __nv_bfloat16 *)x, out, rows, cols);
    else argext_kernel<__nv_bfloat16, false><<<g, 256, 0, st>>>((const __nv_bfloat16 *)x, out, rows, cols);
  } else if (dt == NKB_F16) {
    if (is_max) argext_kernel<__half, true><<<g, 256, 0, st>>>((const __half *)x, out, rows, cols);
    else argext_kernel<__half, false><<<g, 256, 0, st>>>((const __half *)x, out, rows, cols);
  } else {
    return fail(NKB_ERR_UNSUPPORTED, "argmax_rows: dtype not supported");
  }
  return launch_status("argmax_rows");
}

// ---------------------------------------------------------------------------
// generic reduce: out[o] = reduce_{i} view[o, i] over a strided view split
// into outer axes (kept) and inner axes (reduced).  HLO reduce with
// computation add/maximum/minimum/multiply (reference core/ops/reduce.py:14-92).
// ---------------------------------------------------------------------------
constexpr int kRR = 4;
struct ReduceParams {
  const void *in;
  void *out;
  int in_dtype, out_dtype, comp, ro, ri, is_float;
  int64_t n_outer, n_inner, off;
  int64_t oshape[kRR], ostr[kRR], ishape[kRR], istr[kRR];
  float init;
};

__device__ __forceinline__ float fcombine(int comp, float a, float b) {
  switch (comp) {
    case 0: return a + b;
    case 1: return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
    case 2: return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b);
    default: return a * b;
  }
}
__device__ __forceinline__ int32_t icombine(int comp, int32_t a, int32_t b) {
  switch (comp) {
    case 0: return (int32_t)((uint32_t)a + (uint32_t)b);
    case 1: return max(a, b);
    case 2: return min(a, b);
    default: return (int32_t)((uint32_t)a * (uint32_t)b);
  }
}

// WARPS_PER_OUT warps cooperate on one output element.
template <int WARPS_PER_OUT>
__global__ void __launch_bounds__(256) reduce_kernel(const __grid_constant__ ReduceParams p) {
  constexpr int OPB = 8 / WARPS_PER_OUT;  // outputs per block
  __shared__ uint32_t smem[8];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int slot = warp / WARPS_PER_OUT, wi = warp % WARPS_PER_OUT;
  for (int64_t o0 = (int64_t)blockIdx.x * OPB; o0 < p.n_outer; o0 += (int64_t)gridDim.x * OPB) {
    const int64_t o = o0 + slot;
    const bool active = o < p.n_outer;
    int64_t base = p.off;
    if (active) {
      int64_t rem = o;
      for (int d = p.ro - 1; d >= 0; --d) {
        const int64_t q = rem / p.oshape[d];
        base += (rem - q * p.oshape[d]) * p.ostr[d];
        rem = q;
      }
    }
    float facc = p.init;
    int32_t iacc = (int32_t)p.init;
    if (active) {
      for (int64_t i = (int64_t)wi * 32 + lane; i < p.n_inner; i += 32 * WARPS_PER_OUT) {
        int64_t rem = i, offs = base;
        for (int d = p.ri - 1; d >= 0; --d) {
          const int64_t q = rem / p.ishape[d];
          offs += (rem - q * p.ishape[d]) * p.istr[d];
          rem = q;
        }
        const uint32_t raw = load_as_reg(p.in, offs, p.in_dtype);
        if (p.is_float) facc = fcombine(p.comp, facc, __uint_as_float(raw));
        else iacc = icombine(p.comp, iacc, (int32_t)raw);
      }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      if (p.is_float) facc = fcombine(p.comp, facc, __shfl_xor_sync(0xffffffffu, facc, s));
      else iacc = icombine(p.comp, iacc, __shfl_xor_sync(0xffffffffu, iacc, s));
    }
    if (WARPS_PER_OUT > 1) {
      __syncthreads();
      if (lane == 0) smem[warp] = p.is_float ? __float_as_uint(facc) : (uint32_t)iacc;
      __syncthreads();
      if (wi == 0 && lane == 0) {
        for (int k = 1; k < WARPS_PER_OUT; ++k) {
          const uint32_t v = smem[warp + k];
          if (p.is_float) facc = fcombine(p.comp, facc, __uint_as_float(v));
          else iacc = icombine(p.comp, iacc, (int32_t)v);
        }
      }
    }
    if (active && wi == 0 && lane == 0)
      store_from_reg(p.out, o, p.out_dtype, p.is_float ? __float_as_uint(facc) : (uint32_t)iacc);
  }
}

// ---- plan steps -------------------------------------------------------------
// "softmax_rows": ptrs x, y; ints rows cols x_dtype y_dtype
int softmax_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() != 4) return fail(NKB_ERR_PLAN, "softmax_rows: bad parameters");
  return NKB_OK;
}
int softmax_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  return softmax_any(a.ptrs[0], (int)q[2], a.ptrs[1], (int)q[3], q[0], q[1], a.stream, a.device);
}

// "rmsnorm_rows": ptrs x r w y hsum (r/hsum may be unused per flags);
// ints rows cols dtype w_dtype has_res has_sum [in_block_rows in_block_stride];
// floats eps.  Without the last two the input rows are dense.
int rmsnorm_check(const Step &s) {
  if (s.buf_ids.size() != 5 || (s.ints.size() != 6 && s.ints.size() != 8) || s.floats.size() != 1)
    return fail(NKB_ERR_PLAN, "rmsnorm_rows: bad parameters");
  return NKB_OK;
}
int rmsnorm_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  const bool blocks = q.size() == 8;
  return rmsnorm_any(a.ptrs[0], q[4] ? a.ptrs[1] : nullptr, a.ptrs[2], a.ptrs[3], q[5] ? a.ptrs[4] : nullptr,
                     (int)q[2], (int)q[3], q[0], q[1], a.step->floats[0], a.stream, a.device,
                     blocks ? q[6] : q[0], blocks ? q[7] : q[0] * q[1]);
}

// "rmsnorm_rope_rows": ptrs x w y cos sin pos (pos unused when has_pos = 0);
// ints rows cols w_dtype in_block_rows in_block_stride table_stride has_pos
//      pos_dtype table_rows S H per_token; floats eps.  x, y, cos, sin bf16.
// Two row sets (6 more ptrs, 12 more ints, the same cols, weight dtype and
// eps) run in one launch: the planner merges adjacent independent steps.
int rmsnorm_rope_check(const Step &s) {
  const size_t n = s.ints.size() / 12;
  if ((n != 1 && n != 2) || s.ints.size() != 12 * n || s.buf_ids.size() != 6 * n || s.floats.size() != 1)
    return fail(NKB_ERR_PLAN, "rmsnorm_rope_rows: bad parameters");
  if (n == 2 && (s.ints[1] != s.ints[13] || s.ints[2] != s.ints[14]))
    return fail(NKB_ERR_PLAN, "rmsnorm_rope_rows: merged row sets differ in width or weight dtype");
  return NKB_OK;
}
int rmsnorm_rope_launch(const LaunchArgs &a) {
  const auto &all = a.step->ints;
  RopeLaunch L;
  L.nseg = (int)(all.size() / 12);
  L.cols = (int)all[1];
  L.eps = a.step->floats[0];
  for (int i = 0; i < L.nseg; ++i) {
    const int64_t *q = all.data() + 12 * i;
    void *const *pp = a.ptrs + 6 * i;
    RopeRows rp;
    rp.cos = static_cast<const __nv_bfloat16 *>(pp[3]);
    rp.sin = static_cast<const __nv_bfloat16 *>(pp[4]);
    rp.tstride = q[5];
    rp.pos = q[6] ? pp[5] : nullptr;
    rp.pos_dt = (int)q[7];
    rp.T = q[8];
    rp.S = q[9];
    rp.H = q[10];
    rp.per_token = (int)q[11];
    if (int e = rope_seg(pp[0], pp[1], pp[2], (int)q[2], q[0], q[1], q[3], q[4], rp, a.device, &L.seg[i])) return e;
  }
  return rope_launch(L, (int)all[2], a.stream, a.pdl);
}

// "argmax_rows": ptrs x out; ints rows cols dtype is_max
int argext_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() != 4) return fail(NKB_ERR_PLAN, "argmax_rows: bad parameters");
  return NKB_OK;
}
int argext_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  return argext_any(a.ptrs[0], (int)q[2], static_cast<int32_t *>(a.ptrs[1]), q[0], q[1], q[3] != 0, a.stream,
                    a.device);
}

// "reduce": ptrs in out; ints in_dtype out_dtype comp ro ri off n_outer n_inner
//           oshape[ro] ostr[ro] ishape[ri] istr[ri]; floats init
int reduce_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() < 8 || s.floats.size() != 1)
    return fail(NKB_ERR_PLAN, "reduce: bad parameters");
  const int64_t ro = s.ints[3], ri = s.ints[4];
  if (ro < 0 || ro > kRR || ri < 1 || ri > kRR) return fail(NKB_ERR_UNSUPPORTED, "reduce: rank out of range");
  if ((int64_t)s.ints.size() != 8 + 2 * ro + 2 * ri) return fail(NKB_ERR_PLAN, "reduce: parameter count");
  return NKB_OK;
}
int reduce_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  ReduceParams p;
  memset(&p, 0, sizeof(p));
  p.in = a.ptrs[0];
  p.out = a.ptrs[1];
  p.in_dtype = (int)q[0];
  p.out_dtype = (int)q[1];
  p.comp = (int)q[2];
  p.ro = (int)q[3];
  p.ri = (int)q[4];
  p.off = q[5];
  p.n_outer = q[6];
  p.n_inner = q[7];
  int k = 8;
  for (int d = 0; d < p.ro; ++d) p.oshape[d] = q[k++];
  for (int d = 0; d < p.ro; ++d) p.ostr[d] = q[k++];
  for (int d = 0; d < p.ri; ++d) p.ishape[d] = q[k++];
  for (int d = 0; d < p.ri; ++d) p.istr[d] = q[k++];
  p.is_float = dtype_is_float(p.in_dtype);
  p.init = a.step->floats[0];
  if (p.n_outer == 0) return NKB_OK;
  const int64_t cap = (int64_t)num_sms(a.device) * 16;
  if (p.n_inner >= 4096) {
    reduce_kernel<8><<<(unsigned)std::min<int64_t>(p.n_outer, cap), 256, 0, a.stream>>>(p);
  } else {
    reduce_kernel<1><<<(unsigned)std::min<int64_t>((p.n_outer + 7) / 8, cap), 256, 0, a.stream>>>(p);
  }
  return launch_status("reduce_kernel");
}

}  // namespace rows

NKB_REGISTER_KERNEL("softmax_rows", rows::softmax_launch, rows::softmax_check);
NKB_REGISTER_KERNEL("rmsnorm_rows", rows::rmsnorm_launch, rows::rmsnorm_check);
NKB_REGISTER_KERNEL("rmsnorm_rope_rows", rows::rmsnorm_rope_launch, rows::rmsnorm_rope_check);
NKB_REGISTER_KERNEL("argmax_rows", rows::argext_launch, rows::argext_check);
NKB_REGISTER_KERNEL("reduce", rows::reduce_launch, rows::reduce_check);

}  // namespace nkb

extern "C" int nkb_softmax_rows(const void *x, int x_dtype, void *out, int out_dtype, int64_t rows, int64_t cols,
                                void *stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  return nkb::rows::softmax_any(x, x_dtype, out, out_dtype, rows, cols, static_cast<cudaStream_t>(stream), dev);
}

extern "C" int nkb_rmsnorm_rows(const void *x, const void *r, const void *w, void *out, void *sum_out, int dtype,
                                int w_dtype, int64_t rows, int64_t cols, float eps, void *stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  return nkb::rows::rmsnorm_any(x, r, w, out, sum_out, dtype, w_dtype, rows, cols, eps,
                                static_cast<cudaStream_t>(stream), dev, rows, rows * cols);
}
