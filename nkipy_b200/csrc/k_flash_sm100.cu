// Fused causal attention (prefill) on the 5th-generation tensor cores
// (sm_100a): the traced composition
//   scores = q @ k^T ; scores / sqrt(d) ; + causal mask ; softmax ; @ v
// of examples/models/qwen3_embedding/kernels/attention.py:85-95 and
// examples/models/qwen3/kernels/attention.py:119-140, without materialising
// the S x S scores (online softmax, fp32 statistics), for head_dim 128.
//
// One CTA = two tiles (A, B) of 128 query rows of one (batch, head); GQA
// query head h reads kv head h / (H / Hkv).  18 warps:
//   warp 16      TMA producer: Q_A, Q_B once, then K and V blocks of 128 keys
//                (128B-swizzled, two 64-column boxes) into a 2-stage ring;
//   warp 17      TMEM owner and MMA issuer (one thread);
//   warps 0-7    softmax of tile A, warps 8-15 of tile B: two threads per query
//                row (64 keys each) read the scores from TMEM, mask, agree on
//                the row maximum through shared memory, write exp2 of the
//                scaled scores back into TMEM as bf16 P, and at the end
//                normalise their halves of the O row into the staging buffer
//                for the TMA store.
// Tensor-core products per key block j, in issue order (M = 128, K = 128):
//   S_A = Q_A K_j^T, S_B = Q_B K_j^T   (A, B K-major in shared memory)
//   O_A += P_A V_j, O_B += P_B V_j     (A = P in TMEM, B = V MN-major)
// issued as S_A(0) S_B(0) PV_A(0) S_A(1) PV_B(0) S_B(1) PV_A(1) ..., so one
// tile's softmax overlaps the other tile's products.  TMEM: S_A, S_B, O_A, O_B
// (4 x 128 columns).  The running maximum is only raised when a row's new
// maximum exceeds it by more than 2^8 (log2 units): O and the row sum are
// then rescaled; otherwise the stale maximum keeps exp2 values below 256,
// and the final division is exact either way.  Every wait is bounded.

#include "sm100.cuh"

namespace nkb {
namespace fa {

using namespace sm100;

constexpr int D = 128, BM = 128, BN = 128;
constexpr int HALF = BM * 64 * 2;  // one 128-row x 64-column bf16 box (16 KB)
constexpr int TILE = 2 * HALF;     // 128 x 128 bf16 (32 KB)
constexpr int W_PROD = 16, W_MMA = 17, THREADS = 18 * 32, SM_THREADS = 256;  // softmax threads per tile
constexpr uint32_t T_SA = 0, T_SB = 128, T_OA = 256, T_OB = 384, TMEM_COLS = 512;
// Q_A | Q_B | stage 0 (K, V) | stage 1 (K, V) | row maxima [parity][tile][half][row] | barriers
constexpr int OFF_Q = 0, OFF_KV = 2 * TILE, OFF_MX = OFF_KV + 2 * 2 * TILE, OFF_BAR = OFF_MX + 2 * 2 * 2 * BM * 4;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr float RESCALE = 8.f;  // log2 headroom before the maximum is raised

__device__ int g_error = 0;

struct Params {
  int B, H, Hkv, Sq, Skv, shift;  // shift = Skv - Sq: query row r sees keys <= r + shift
  int causal;
  float scale_log2;  // softmax scale * log2(e)
};

__device__ __forceinline__ bool wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return sm100::mbar_wait(bar, parity, abort_flag, &g_error);
}
__device__ __forceinline__ bool wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return __all_sync(0xffffffffu, wait(bar, parity, abort_flag));
}
// named barrier `id` over one tile's softmax threads; true iff `ok` held for all of them
__device__ __forceinline__ bool group_and(int id, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id), "n"(SM_THREADS)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(SM_THREADS) : "memory"); }
// 2^x on the special-function unit (PTX ex2.approx, relative error ~2^-22; -inf -> 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk) {
  return smem_desc(base + (kk >> 2) * HALF + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int kk) { return smem_desc(base + kk * 2048, HALF, 1024); }
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (c >> 6) * HALF + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2;
}

// key blocks a tile of query rows [q0, q0 + 128) attends to
__device__ __forceinline__ int tile_blocks(const Params &p, int q0) {
  if (q0 >= p.Sq) return 0;
  int last = p.Skv - 1;
  if (p.causal) last = min(last, q0 + BM - 1 + p.shift);
  return last < 0 ? 0 : last / BN + 1;
}

__global__ void __launch_bounds__(THREADS, 1)
    fa_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                 const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mo,
                 const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  float *sMx = reinterpret_cast<float *>(smem + OFF_MX);
  uint64_t *q_full = bars, *k_full = bars + 1, *v_full = bars + 3, *kv_empty = bars + 5;
  uint64_t *s_full = bars + 7, *p_ready = bars + 9, *o_done = bars + 11;  // [tile]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 13);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int npairs = (p.Sq + 2 * BM - 1) / (2 * BM);
  const int pair = npairs - 1 - (int)blockIdx.x;  // longest (causal) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.H / p.Hkv);
  const int q0 = pair * 2 * BM;
  const int nb[2] = {tile_blocks(p, q0), tile_blocks(p, q0 + BM)};
  const int nblk = max(nb[0], nb[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], SM_THREADS);
      mbar_init(&o_done[s], 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == W_PROD && lane == 0) {
    prefetch_map(&mq);
    prefetch_map(&mk);
    prefetch_map(&mv);
    prefetch_map(&mo);
  }
  if (warp == W_MMA) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == W_PROD) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && nblk > 0) {
      mbar_expect_tx(q_full, 2 * TILE);
      for (int t = 0; t < 2; ++t)
        for (int j = 0; j < 2; ++j) tma_load_4d(smem + OFF_Q + t * TILE + j * HALF, &mq, q_full, j * 64, q0 + t * BM, h, b);
      for (int c = 0; c < nblk; ++c) {
        const int st = c & 1;
        if (!wait(&kv_empty[st], ((c >> 1) & 1) ^ 1, abort_flag)) break;
        uint8_t *kt = smem + OFF_KV + st * 2 * TILE, *vt = kt + TILE;
        mbar_expect_tx(&k_full[st], TILE);
        for (int j = 0; j < 2; ++j) tma_load_4d(kt + j * HALF, &mk, &k_full[st], j * 64, c * BN, hk, b);
        mbar_expect_tx(&v_full[st], TILE);
        for (int j = 0; j < 2; ++j) tma_load_4d(vt + j * HALF, &mv, &v_full[st], j * 64, c * BN, hk, b);
      }
    }
  } else if (warp == W_MMA) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, BN, 0, 0), ID_O = idesc_bf16(128, D, 0, 1);
      const uint32_t qa = smem_u32(smem + OFF_Q), qb = qa + TILE;
      const uint32_t ts[2] = {tmem + T_SA, tmem + T_SB}, to[2] = {tmem + T_OA, tmem + T_OB};
      const uint32_t qt[2] = {qa, qb};
      auto qk = [&](int t, int c) {  // S_t = Q_t K_c^T
        const uint32_t kt = smem_u32(smem + OFF_KV + (c & 1) * 2 * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) umma_f16(ts[t], desc_k(qt[t], kk), desc_k(kt, kk), ID_S, kk > 0);
        umma_commit(&s_full[t]);
      };
      auto pv = [&](int t, int c) {  // O_t += P_t V_c
        const uint32_t vt = smem_u32(smem + OFF_KV + (c & 1) * 2 * TILE + TILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) umma_f16_ts(to[t], ts[t] + kk * 8, desc_mn(vt, kk), ID_O, (c > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      bool ok = wait(q_full, 0, abort_flag) && wait(&k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nb[t] > 0) qk(t, 0);
      }
      for (int c = 0; ok && c < nblk; ++c) {
        const int st = c & 1;
        const bool more = c + 1 < nblk;
        bool next_k = false;
        if (!wait(&v_full[st], (c >> 1) & 1, abort_flag)) break;
        for (int t = 0; t < 2; ++t) {
          if (c < nb[t]) {
            if (!wait(&p_ready[t], c & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv(t, c);
          }
          if (more && c + 1 < nb[t]) {
            if (!next_k) {
              if (!wait(&k_full[st ^ 1], ((c + 1) >> 1) & 1, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              next_k = true;
            }
            qk(t, c + 1);
          }
        }
        if (ok) umma_commit(&kv_empty[st]);
      }
    }
  } else {
    // ------- softmax and epilogue: tile t, row r = 32*(warp%4) + lane, keys/columns of half hf -------
    const int t = warp >> 3, hf = (warp >> 2) & 1, quad = warp & 3, r = quad * 32 + lane;
    const int row = q0 + t * BM + r, bar_id = 1 + t;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t s_col = (t ? T_SB : T_SA) + hf * 64, o_col = (t ? T_OB : T_OA) + hf * 64;
    const uint32_t p_col = (t ? T_SB : T_SA) + hf * 32;  // P columns of this half's keys
    float m = -INFINITY, l = 0.f;  // running (possibly stale) maximum in log2 units, partial row sum
    bool ok = true;
    for (int c = 0; c < nb[t]; ++c) {
      // one decision for the tile's softmax warps (they meet at named barriers)
      if (!group_and(bar_id, ok && wait_warp(&s_full[t], c & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = c * BN + hf * 64;
      // keys of this half visible to the row: [k0, k0 + lim)
      int lim = min(64, p.Skv - k0);
      if (p.causal) lim = min(lim, row + p.shift - k0 + 1);
      uint32_t v[64];
      tmem_ld32_nw(lane_base + s_col, v);
      tmem_ld32_nw(lane_base + s_col + 32, v + 32);
      tmem_ld_wait();
      if (__any_sync(0xffffffffu, lim < 64)) {  // diagonal or last block
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (j >= lim) v[j] = 0xff800000u;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 64; ++j) mx4[j & 3] = fmaxf(mx4[j & 3], __uint_as_float(v[j]));
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // the row maximum of both halves (double-buffered by block parity)
      float *mslot = sMx + ((c & 1) * 2 + t) * 2 * BM;
      mslot[hf * BM + r] = mx;
      group_sync(bar_id);
      mx = fmaxf(mx, mslot[(hf ^ 1) * BM + r]);
      mx = mx == -INFINITY ? -INFINITY : mx * p.scale_log2;
      // raise the running maximum only when the headroom is used up (the same
      // decision in both halves of a row, and warp-uniform for the TMEM rescale)
      const bool raise = mx > m + RESCALE;
      if (__any_sync(0xffffffffu, raise)) {
        const float m_new = raise ? mx : m;
        const float alpha = (m == -INFINITY || !raise) ? (m == -INFINITY ? 0.f : 1.f) : ex2(m - m_new);
        if (c > 0) {
          // O holds the products of blocks < c: wait for the last one, scale this half in TMEM
          ok = wait_warp(&o_done[t], (c - 1) & 1, abort_flag);
          if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int g = 0; g < 4; ++g) {
              uint32_t o[16];
              tmem_ld16(lane_base + o_col + g * 16, o);
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
              tmem_st16(lane_base + o_col + g * 16, o);
            }
            tmem_st_wait();
          }
        }
        l *= alpha;
        m = m_new;
      }
      // P = exp2(s * scale - m) in bf16, packed in place (P column c holds keys 2c, 2c+1)
      const float mm = m == -INFINITY ? 0.f : m;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        const float e0 = ex2(fmaf(__uint_as_float(v[j]), p.scale_log2, -mm));
        const float e1 = ex2(fmaf(__uint_as_float(v[j + 1]), p.scale_log2, -mm));
        l4[(j >> 1) & 3] += e0 + e1;
        v[j / 2] = pack_bf16(e0, e1);
      }
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      // both halves have read their scores (the exchange above), so P may
      // overwrite them; each half writes its own 32 P columns
      tmem_st16(lane_base + p_col, v);
      tmem_st16(lane_base + p_col + 16, v + 16);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_ready[t]);
    }
    // epilogue: O / l -> bf16 -> staging (the Q tile, consumed) -> TMA store
    if (nb[t] > 0 && group_and(bar_id, ok && wait_warp(&o_done[t], (nb[t] - 1) & 1, abort_flag))) {
      tc_fence_after();
      float *lslot = sMx;  // the maxima are no longer needed: reuse for the row sums
      lslot[(t * 2 + hf) * BM + r] = l;
      group_sync(bar_id);
      const float lt = l + lslot[(t * 2 + (hf ^ 1)) * BM + r];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint8_t *stg = smem + OFF_Q + t * TILE;
#pragma unroll 1
      for (int g = 0; g < 2; ++g) {
        uint32_t o[32];
        tmem_ld32(lane_base + o_col + g * 32, o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 w;
          w.x = pack_bf16(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
          w.y = pack_bf16(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
          w.z = pack_bf16(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
          w.w = pack_bf16(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
          *reinterpret_cast<uint4 *>(stg + swz_off(r, hf * 64 + g * 32 + i * 8)) = w;
        }
      }
      fence_proxy_async_smem();
      group_sync(bar_id);
      if (hf == 0 && quad == 0 && lane == 0) {
        for (int j = 0; j < 2; ++j) tma_store_4d(&mo, stg + j * HALF, j * 64, q0 + t * BM, h, b);
        bulk_commit();
        bulk_wait<0>();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && warp == W_PROD && lane == 0) {
    const long long t0 = clock64();
    while (clock64() - t0 < 2000000) {
    }
  }
  __syncthreads();
  if (warp == W_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

struct Operand {
  const void *ptr;
  int64_t sb, sh, ss;  // element strides of batch, head, position
};

// (d, s, h, b) tensor map with 64 x 128 boxes; unit dims get a valid stride
static int make_map(CUtensorMap *m, const Operand &x, int64_t B, int64_t H, int64_t S) {
  const int64_t ss = x.ss, sh = H > 1 ? x.sh : ss * S, sb = B > 1 ? x.sb : sh * H;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)ss, (uint64_t)sh, (uint64_t)sb};
  const uint32_t box[4] = {64, BM, 1, 1};
  return make_bf16_map(m, x.ptr, 4, dims, strides, box);
}

}  // namespace fa

// Can the tcgen05 kernel take this attention?  (head_dim 128, positive
// position strides, 16-byte aligned bases; strides are checked by the step)
bool fa_tc_eligible(int D, int64_t qs, int64_t ks, int64_t vs, int64_t os) {
  return D == fa::D && qs > 0 && ks > 0 && vs > 0 && os > 0;
}

int fa_tc_launch(const void *q, const void *k, const void *v, void *o, int B, int H, int Hkv, int Sq, int Skv,
                 int causal, float scale, const int64_t *qst, const int64_t *kst, const int64_t *vst,
                 const int64_t *ost, cudaStream_t st, int device) {
  using namespace fa;
  static ContextOnce attr;
  if (int s = attr.run(device, []() -> int {
        NKB_CUDA_TRY(cudaFuncSetAttribute(fa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        return NKB_OK;
      }))
    return s;
  CUtensorMap mq, mk, mv, mo;
  if (int s = make_map(&mq, Operand{q, qst[0], qst[1], qst[2]}, B, H, Sq)) return s;
  if (int s = make_map(&mk, Operand{k, kst[0], kst[1], kst[2]}, B, Hkv, Skv)) return s;
  if (int s = make_map(&mv, Operand{v, vst[0], vst[1], vst[2]}, B, Hkv, Skv)) return s;
  if (int s = make_map(&mo, Operand{o, ost[0], ost[1], ost[2]}, B, H, Sq)) return s;
  Params p;
  p.B = B;
  p.H = H;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.shift = Skv - Sq;
  p.causal = causal;
  p.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((Sq + 2 * BM - 1) / (2 * BM), H, B);
  if (grid.y > 65535 || grid.z > 65535) return fail(NKB_ERR_UNSUPPORTED, "flash_attn: too many heads or batches");
  fa_tc_kernel<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, mo, p);
  return launch_status("fa_tc_kernel");
}

int fa_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, fa::g_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(fa::g_error, &zero, sizeof(int)));
  return NKB_OK;
}

}  // namespace nkb
