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
#include <cstdlib>

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

// ---------------------------------------------------------------------------
// k <= 32: one pass over the row.  A row is cut into `parts` ranges, one CTA
// (256 threads) each; every thread keeps the KL largest keys it has seen in a
// sorted register list (one compare against the list's last key rejects
// almost every element), reading the row 16 bytes at a time.  The CTA then
// merges its 256 lists (k rounds of warp max + pop per warp, then across the
// eight warps); with several parts a second kernel merges the parts' lists.
// ---------------------------------------------------------------------------
constexpr int kPartThreads = 256;

template <int KL>
__device__ __forceinline__ void list_insert(uint64_t (&lst)[KL], uint64_t key) {
  if (key > lst[KL - 1]) {
#pragma unroll
    for (int j = KL - 1; j > 0; --j) lst[j] = key > lst[j - 1] ? lst[j - 1] : (key > lst[j] ? key : lst[j]);
    lst[0] = key > lst[0] ? key : lst[0];
  }
}

// Top `k` keys over the lists of the warp's lanes (k <= KL); lane 0 ends with
// them in out[0..k).  Lists are sorted descending; a lane pops its head when it wins.
template <int KL>
__device__ __forceinline__ void warp_merge(uint64_t (&lst)[KL], int k, uint64_t *out) {
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < k; ++r) {
    const uint64_t best = warp_max64(lst[0]);
    if (lane == 0) out[r] = best;
    if (lst[0] == best && best != 0) {  // keys are distinct: exactly one lane owns it
#pragma unroll
      for (int j = 0; j < KL - 1; ++j) lst[j] = lst[j + 1];
      lst[KL - 1] = 0;
    }
  }
}

__device__ __forceinline__ uint64_t make_key(uint32_t img, int64_t c) {
  return ((uint64_t)img << 32) | (uint32_t)~(uint32_t)c;
}

__device__ __forceinline__ void emit(const void *x, int64_t base, int64_t cols, int esize, uint64_t key, void *vals,
                                     uint32_t *idx, int64_t o) {
  uint32_t col = ~(uint32_t)(key & 0xffffffffu);
  if (col >= cols) col = 0;  // only an empty-list sentinel (never reached when k <= cols) lies outside the row
  idx[o] = col;
  const uint8_t *src = static_cast<const uint8_t *>(x) + (base + col) * esize;
  uint8_t *dst = static_cast<uint8_t *>(vals) + o * esize;
  for (int b = 0; b < esize; ++b) dst[b] = src[b];
}

constexpr int RES_V = 8;  // 16-byte vectors per thread in the register-resident path (64 registers: 4 CTAs per SM)
constexpr int kCand = kPartThreads;  // candidate keys a part may collect (one per thread to rank)

// The kk-th largest (kk <= 32) of the block's per-thread values; every thread
// of the block calls it and gets the same result.
__device__ uint32_t block_kth_largest(uint32_t v, int kk) {
  __shared__ uint32_t s_top[kPartThreads / 32][32];
  __shared__ uint32_t s_res;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // each warp: its kk largest, popping one lane (the lowest among equals) per round
  for (int r = 0; r < kk; ++r) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, v);
    const int win = __ffs(__ballot_sync(0xffffffffu, v == m)) - 1;
    if (lane == 0) s_top[warp][r] = m;
    if (lane == win) v = 0;
  }
  __syncthreads();
  if (warp == 0) {
    // merge the warps' sorted lists: lane w < 8 walks list w
    int ptr = 0;
    uint32_t m = 0;
    for (int r = 0; r < kk; ++r) {
      const uint32_t head = (lane < kPartThreads / 32 && ptr < kk) ? s_top[lane][ptr] : 0u;
      m = __reduce_max_sync(0xffffffffu, head);
      const unsigned own = __ballot_sync(0xffffffffu, lane < kPartThreads / 32 && ptr < kk && head == m);
      if (lane == __ffs(own) - 1) ++ptr;
    }
    if (lane == 0) s_res = m;
  }
  __syncthreads();
  return s_res;
}

template <int KL>
__global__ void __launch_bounds__(kPartThreads) topk_part_kernel(const void *__restrict__ x, int dt, int64_t rows,
                                                                 int64_t cols, int parts, int64_t part_len, int k,
                                                                 int esize, int vec, int resident,
                                                                 uint64_t *__restrict__ ws,
                                                                 void *__restrict__ vals, uint32_t *__restrict__ idx) {
  __shared__ uint64_t s_cand[kPartThreads / 32][KL];
  // the merge kernel may launch once every part CTA has started (it waits for
  // this grid to finish before reading the lists); the last wave is partial,
  // so its CTAs find free slots
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x / parts;
  const int part = (int)(blockIdx.x % parts);
  if (row >= rows) return;
  const int64_t base = row * cols;
  const int64_t c0 = (int64_t)part * part_len, c1 = min(cols, c0 + part_len);
  uint64_t lst[KL];
#pragma unroll
  for (int j = 0; j < KL; ++j) lst[j] = 0;
  // A thread sees its columns in increasing order, so an element whose value
  // image is below the image of its list's last key can never enter the list:
  // a 32-bit compare rejects it.  The images of a 16-byte vector are computed
  // branch-free and the warp votes once per vector, so the insert code is
  // skipped by the whole warp unless some lane has a candidate (rare once the
  // lists have filled).
  constexpr int UNROLL = 4;  // 16-byte loads in flight per thread
  const bool flt = dt == NKB_F32 || dt == NKB_BF16 || dt == NKB_F16;
  const uint32_t sx = (dt == NKB_I32) ? 0x80000000u : 0u;  // signed int: flip the sign bit
  auto image = [&](uint32_t bits) -> uint32_t {  // order_bits without a branch
    return bits ^ (flt ? ((uint32_t)((int32_t)bits >> 31) | 0x80000000u) : sx);
  };
  // Loop bounds are taken from the warp's first index, so all 32 lanes run the
  // same iterations (the vote needs every lane); a lane past the end holds no
  // candidate.
  const int64_t wtid = tid & ~31;
  const int kk = parts > 1 ? KL : k;  // a part hands on its full list
  if (resident) {
    // The part fits in registers (at most RES_V 16-byte vectors per thread).
    // Pass 1: each thread's largest value image; T = the kk-th largest of
    // those maxima.  kk threads hold an element at or above T, so every one of
    // the part's kk largest keys has an image >= T: pass 2 inserts only those
    // elements (few), instead of testing every element against a list.
    const int per = vec == 2 ? 8 : 4;
    const int64_t nv = (c1 - c0) / per;
    const uint4 *pv = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(x) + (base + c0) * esize);
    auto images = [&](const uint4 &v, uint32_t (&img)[8]) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (vec == 2) {
          const uint32_t h = (w[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
          img[e] = image(dt == NKB_BF16 ? (h << 16) : __float_as_uint(__half2float(__ushort_as_half((uint16_t)h))));
        } else {
          img[e] = e < 4 ? image(w[e]) : 0u;
        }
      }
    };
    uint4 u[RES_V];
#pragma unroll
    for (int q = 0; q < RES_V; ++q) {
      const int64_t i = tid + (int64_t)q * kPartThreads;
      u[q] = i < nv ? pv[i] : make_uint4(0, 0, 0, 0);
    }
    // k <= 8 (KL == 8): the threshold is the smallest of the eight warps'
    // maxima.  Those are eight distinct elements, so the part's kk <= 8
    // largest keys all have images at or above it.  The elements that reach it
    // (a few dozen on typical rows) are appended to a shared-memory list and
    // each one's rank among them is counted directly: no merge rounds.  More
    // than kCand of them (heavy ties, or a warp without elements) take the
    // list path below.
    __shared__ uint32_t s_wmax[kPartThreads / 32];
    __shared__ uint64_t s_keys[kCand];
    __shared__ int s_n;
    auto append = [&](uint32_t img, int64_t c) {
      const int slot = atomicAdd(&s_n, 1);
      if (slot < kCand) s_keys[slot] = make_key(img, c);
    };
    // every thread: the warps' maxima in, the smallest of them out
    auto warp_threshold = [&](uint32_t tm) -> uint32_t {
      const uint32_t wm = __reduce_max_sync(0xffffffffu, tm);
      if (lane == 0) s_wmax[warp] = wm;
      if (tid == 0) s_n = 0;
      __syncthreads();
      uint32_t t8 = s_wmax[0];
#pragma unroll
      for (int w = 1; w < kPartThreads / 32; ++w) t8 = min(t8, s_wmax[w]);
      return t8;
    };
    // after the appends: rank the candidates and hand on the kk largest; false
    // when there were too many (every thread gets the same answer)
    auto rank_candidates = [&]() -> bool {
      __syncthreads();
      const int n = s_n;
      if (n > kCand) return false;
      if (tid < n) {
        const uint64_t key = s_keys[tid];
        int rank = 0;
        for (int j = 0; j < n; ++j) rank += s_keys[j] > key ? 1 : 0;
        if (parts > 1) {
          if (rank < kk) ws[((int64_t)row * parts + part) * KL + rank] = key;
        } else if (rank < k) {
          emit(x, base, cols, esize, key, vals, idx, row * k + rank);
        }
      }
      return true;
    };
    uint32_t tmax = 0;
#pragma unroll
    for (int q = 0; q < RES_V; ++q) {
      if (tid + (int64_t)q * kPartThreads < nv) {
        uint32_t img[8];
        images(u[q], img);
#pragma unroll
        for (int e = 0; e < 8; ++e) tmax = max(tmax, e < per ? img[e] : 0u);
      }
    }
    for (int64_t c = c0 + nv * per + tid; c < c1; c += kPartThreads)
      tmax = max(tmax, order_bits(load_as_reg(x, base + c, dt), dt));
    if constexpr (KL == 8) {
      const uint32_t T8 = warp_threshold(tmax);
#pragma unroll
      for (int q = 0; q < RES_V; ++q) {
        const int64_t i = tid + (int64_t)q * kPartThreads;
        if (i < nv) {
          uint32_t img[8];
          images(u[q], img);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < per && img[e] >= T8) append(img[e], c0 + i * per + e);
        }
      }
      for (int64_t c = c0 + nv * per + tid; c < c1; c += kPartThreads) {
        const uint32_t img = order_bits(load_as_reg(x, base + c, dt), dt);
        if (img >= T8) append(img, c);
      }
      if (rank_candidates()) return;
    }
    const uint32_t T = block_kth_largest(tmax, kk);
    // every lane runs every q (the vote needs the whole warp); the insert code
    // runs only when some lane of the warp holds a candidate
#pragma unroll
    for (int q = 0; q < RES_V; ++q) {
      const int64_t i = tid + (int64_t)q * kPartThreads;
      const bool valid = i < nv;
      uint32_t img[8];
      images(u[q], img);
      bool cand = false;
#pragma unroll
      for (int e = 0; e < 8; ++e) cand |= valid && e < per && img[e] >= T;
      if (__any_sync(0xffffffffu, cand) && cand) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < per && img[e] >= T) list_insert<KL>(lst, make_key(img[e], c0 + i * per + e));
      }
    }
    for (int64_t c = c0 + nv * per + tid; c < c1; c += kPartThreads) {
      const uint32_t img = order_bits(load_as_reg(x, base + c, dt), dt);
      if (img >= T) list_insert<KL>(lst, make_key(img, c));
    }
  } else if (vec == 2) {  // bf16 / f16 rows, 8 per 16-byte load (c0 and the row start 16-byte aligned)
    const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + base + c0);
    const int64_t n8 = (c1 - c0) / 8;
    for (int64_t ib = wtid; ib < n8; ib += UNROLL * kPartThreads) {
      uint4 u[UNROLL];
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) {
        const int64_t i = ib + lane + q * kPartThreads;
        u[q] = i < n8 ? p[i] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) {
        const int64_t i = ib + lane + q * kPartThreads;
        const bool valid = i < n8;
        const uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
        uint32_t img[8];
        bool cand = false;
        const uint32_t thr = (uint32_t)(lst[KL - 1] >> 32);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t h = (w[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
          const uint32_t bits =
              dt == NKB_BF16 ? (h << 16) : __float_as_uint(__half2float(__ushort_as_half((uint16_t)h)));
          img[e] = image(bits);
          cand |= valid && img[e] >= thr;
        }
        if (__any_sync(0xffffffffu, cand) && valid) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (img[e] >= (uint32_t)(lst[KL - 1] >> 32)) list_insert<KL>(lst, make_key(img[e], c0 + i * 8 + e));
        }
      }
    }
    for (int64_t c = c0 + n8 * 8 + tid; c < c1; c += kPartThreads)
      list_insert<KL>(lst, make_key(order_bits(load_as_reg(x, base + c, dt), dt), c));
  } else if (vec == 4) {  // fp32 / int32 / uint32 rows, 4 per load
    const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint32_t *>(x) + base + c0);
    const int64_t n4 = (c1 - c0) / 4;
    for (int64_t ib = wtid; ib < n4; ib += UNROLL * kPartThreads) {
      uint4 u[UNROLL];
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) {
        const int64_t i = ib + lane + q * kPartThreads;
        u[q] = i < n4 ? p[i] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) {
        const int64_t i = ib + lane + q * kPartThreads;
        const bool valid = i < n4;
        const uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
        uint32_t img[4];
        bool cand = false;
        const uint32_t thr = (uint32_t)(lst[KL - 1] >> 32);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          img[e] = image(w[e]);
          cand |= valid && img[e] >= thr;
        }
        if (__any_sync(0xffffffffu, cand) && valid) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (img[e] >= (uint32_t)(lst[KL - 1] >> 32)) list_insert<KL>(lst, make_key(img[e], c0 + i * 4 + e));
        }
      }
    }
    for (int64_t c = c0 + n4 * 4 + tid; c < c1; c += kPartThreads)
      list_insert<KL>(lst, make_key(order_bits(load_as_reg(x, base + c, dt), dt), c));
  } else {
    for (int64_t c = c0 + tid; c < c1; c += kPartThreads)
      list_insert<KL>(lst, make_key(order_bits(load_as_reg(x, base + c, dt), dt), c));
  }
  warp_merge<KL>(lst, kk, s_cand[warp]);
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int j = 0; j < KL; ++j) lst[j] = (lane < kPartThreads / 32 && j < kk) ? s_cand[lane][j] : 0;
    __shared__ uint64_t s_out[KL];
    warp_merge<KL>(lst, kk, s_out);
    __syncwarp();
    if (parts > 1) {
      if (lane < kk) ws[((int64_t)row * parts + part) * KL + lane] = s_out[lane];
    } else if (lane < k) {
      emit(x, base, cols, esize, s_out[lane], vals, idx, row * k + lane);
    }
  }
}

// one warp per row: the parts' lists (parts * KL keys) -> the row's top k
template <int KL>
__global__ void __launch_bounds__(256, 1) topk_merge_kernel(const void *__restrict__ x, int64_t rows, int64_t cols,
                                                         int parts, int k, int esize,
                                                         const uint64_t *__restrict__ ws, void *__restrict__ vals,
                                                         uint32_t *__restrict__ idx) {
  __shared__ uint64_t s_out[8][KL];
  pdl_wait();  // launched early (programmatic dependent launch): the parts' lists are complete after this
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;  // whole warps leave together
  uint64_t lst[KL];
#pragma unroll
  for (int j = 0; j < KL; ++j) lst[j] = 0;
  const uint64_t *src = ws + row * parts * KL;
  for (int i = lane; i < parts * KL; i += 32) list_insert<KL>(lst, src[i]);
  warp_merge<KL>(lst, k, s_out[warp]);
  __syncwarp();
  if (lane < k) emit(x, row * cols, cols, esize, s_out[warp][lane], vals, idx, row * k + lane);
}

template <int KL>
int topk_parts(const void *x, int dt, void *vals, uint32_t *idx, int64_t rows, int64_t cols, int k, int esize,
               uint64_t *ws, int64_t ws_keys, int parts, cudaStream_t st, int device) {
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
  int vec = 0;
  if (esize == 2 && (dt == NKB_BF16 || dt == NKB_F16) && (xa & 15) == 0 && (cols * 2) % 16 == 0) vec = 2;
  if (esize == 4 && (dt == NKB_F32 || dt == NKB_I32 || dt == NKB_U32) && (xa & 15) == 0 && (cols * 4) % 16 == 0)
    vec = 4;
  // register-resident when a part fits in RES_V vectors per thread (more parts
  // if the workspace has room for their lists)
  int resident = 0;
  if (vec) {
    const int64_t cap = (int64_t)kPartThreads * RES_V * (vec == 2 ? 8 : 4);
    const int64_t need = (cols + cap - 1) / cap;
    if (need <= parts) {
      resident = 1;
    } else if (need <= 64 && ws && ws_keys >= rows * need * KL) {
      parts = (int)need;
      resident = 1;
    }
  }
  int64_t part_len = (cols + parts - 1) / parts;
  part_len = (part_len + 7) / 8 * 8;  // part starts stay 16-byte aligned
  if (resident && part_len > (int64_t)kPartThreads * RES_V * (vec == 2 ? 8 : 4)) resident = 0;
  topk_part_kernel<KL><<<(unsigned)(rows * parts), kPartThreads, 0, st>>>(x, dt, rows, cols, parts, part_len, k, esize,
                                                                          vec, resident, ws, vals, idx);
  if (int e = launch_status("topk_part_kernel")) return e;
  if (parts == 1) return NKB_OK;
  if (cudaError_t e = launch_pdl(true, topk_merge_kernel<KL>, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, x, rows,
                                 cols, parts, k, esize, (const uint64_t *)ws, vals, idx))
    return fail(NKB_ERR_CUDA, std::string("topk_merge_kernel: ") + cudaGetErrorString(e));
  return launch_status("topk_merge_kernel");
}

// Parts per row for the one-pass path: enough CTAs for eight per SM, at least
// 4096 columns per part, at most 64 parts.
int topk_parts_for(int64_t rows, int64_t cols, int sms) {
  if (const char *e = getenv("NKB_TOPK_PARTS")) {  // override (sweeps); bounded like the default
    const int64_t v = atoll(e);
    if (v >= 1) return (int)std::min<int64_t>(std::min<int64_t>(v, 64), std::max<int64_t>(1, cols / 8));
  }
  int64_t p = (8 * (int64_t)sms + rows - 1) / std::max<int64_t>(rows, 1);
  p = std::min<int64_t>(p, std::max<int64_t>(1, cols / 4096));
  return (int)std::max<int64_t>(1, std::min<int64_t>(p, 64));
}

int topk_any(const void *x, int dt, void *vals, uint32_t *idx, int64_t rows, int64_t cols, int64_t k,
             cudaStream_t stream, int device, uint64_t *ws = nullptr, int64_t ws_keys = 0) {
  const int es = dtype_size(dt);
  if (!es || dt == NKB_F8E4M3 || dt == NKB_F8E5M2) return fail(NKB_ERR_UNSUPPORTED, "topk: dtype");
  if (k < 1 || k > cols) return fail(NKB_ERR_INVALID, "topk: k must be in [1, cols]");
  if (cols >= 0xffffffffll) return fail(NKB_ERR_UNSUPPORTED, "topk: rows of 2^32 - 1 or more elements");
  if (rows == 0) return NKB_OK;
  if (k <= 32 && rows <= INT32_MAX / 64) {
    const int KL = k <= 8 ? 8 : k <= 16 ? 16 : 32;
    int parts = topk_parts_for(rows, cols, num_sms(device));
    if (parts > 1 && (!ws || ws_keys < rows * parts * KL)) parts = 1;  // no room for the parts' lists
    if (KL == 8) return topk_parts<8>(x, dt, vals, idx, rows, cols, (int)k, es, ws, ws_keys, parts, stream, device);
    if (KL == 16) return topk_parts<16>(x, dt, vals, idx, rows, cols, (int)k, es, ws, ws_keys, parts, stream, device);
    return topk_parts<32>(x, dt, vals, idx, rows, cols, (int)k, es, ws, ws_keys, parts, stream, device);
  }
  const bool staged = cols <= kSmemCols;
  const size_t smem = staged ? (size_t)cols * 4 : 0;
  if (smem > 48 * 1024)
    NKB_CUDA_TRY(cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t cap = (int64_t)num_sms(device) * (staged && smem > 64 * 1024 ? 1 : 2);
  topk_rows_kernel<<<(unsigned)std::min<int64_t>(rows, cap), kThreads, smem, stream>>>(x, dt, vals, idx, rows, cols,
                                                                                        (int)k, es, staged);
  return launch_status("topk_rows_kernel");
}

// "topk_rows": ptrs x values indices [ws]; ints rows cols k dtype [ws_keys]
// (ws: room for the per-part key lists of the one-pass path, ws_keys uint64 keys)
int check(const Step &s) {
  if (!((s.buf_ids.size() == 3 && s.ints.size() == 4) || (s.buf_ids.size() == 4 && s.ints.size() == 5)))
    return fail(NKB_ERR_PLAN, "topk_rows: bad parameters");
  if (s.ints[2] < 1 || s.ints[2] > s.ints[1]) return fail(NKB_ERR_PLAN, "topk_rows: k out of range");
  return NKB_OK;
}
int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  const bool has_ws = q.size() == 5;
  return topk_any(a.ptrs[0], (int)q[3], a.ptrs[1], static_cast<uint32_t *>(a.ptrs[2]), q[0], q[1], q[2], a.stream,
                  a.device, has_ws ? static_cast<uint64_t *>(a.ptrs[3]) : nullptr, has_ws ? q[4] : 0);
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
