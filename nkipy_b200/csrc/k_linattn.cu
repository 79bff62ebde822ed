// Chunked causal linear attention on the 5th-generation tensor cores
// (sm_100a).  Feature map phi = elu + 1, fp32 running state.  For a block of
// tokens starting at t0:
//   S = sum_{s < t0} phi(k_s) v_s^T,   z = sum_{s < t0} phi(k_s)
//   out_t = (sum_{t0 <= s <= t} (phi(q_t).phi(k_s)) v_s + phi(q_t) S) /
//           (sum_{t0 <= s <= t}  phi(q_t).phi(k_s)       + phi(q_t).z)
// This is the kernel body nkipy_b200/workloads.py:chunked_linear_attention_kernel
// (chunk 64), whose per-step state update follows
// examples/linear_attention/deltanet.py; the kernel evaluates the same sums
// in blocks of 128 tokens (the block length only changes the fp32 summation
// order).
//
// One CTA per (batch*head, segment of the sequence), 22 warps:
//   warp 20      TMA producer: Q, K, V blocks (128 tokens x 128, bf16,
//                128B-swizzled) into a 2-stage ring;
//   warp 21      TMEM owner and MMA issuer (one thread);
//   warps 12-19  feature map phi, in place on the Q and K tiles;
//   warps 0-3    score epilogue: P = phi(Q) phi(K)^T from TMEM, causal mask,
//                row sums + phi(q_t).z -> 1 / denominator, bf16 P written over
//                the consumed Q tile;
//   warps 4-11   two teams of four: state conversion (S^T fp32 -> bf16 TMEM
//                operand, z -> bf16 hi/lo operand tile) and output epilogue
//                (O^T from TMEM x 1/denominator -> swizzled staging -> TMA
//                store), team 0 on tokens 0-63 of a block, team 1 on 64-127.
// Tensor-core products per block (M = 128, K = 128, bf16 in, fp32 accumulate):
//   P    = phi(Q) phi(K)^T        N 128   A, B K-major in shared memory
//   O^T  = S^T phi(Q)^T           N 128   A = bf16 copy of S^T in TMEM
//   qz   = phi(Q) [z_hi z_lo]     N 16    phi(q_t).z in two bf16 halves
//   S^T += V^T phi(K)             N 128   A, B MN-major
//   z   += phi(K)^T 1             N 16    key sums against a ones tile
//   O^T += V^T P^T                N 128   A MN-major, B = P K-major
// The fp32 state S^T and key sum z stay in TMEM for the whole segment.  When
// the sequence is split into segments (few heads, long sequences) a
// state-only pass writes each segment's totals to a workspace, a scan turns
// those into exclusive prefixes, and the output pass seeds its state from
// them.  Every wait is bounded; on expiry the CTA raises the device error
// flag and winds down.

#include <mutex>

#include "sm100.cuh"

namespace nkb {
namespace linattn {

using namespace sm100;

constexpr int TB = 128;            // tokens per block
constexpr int D = 128;             // head dimension
constexpr int HALF = TB * 64 * 2;  // one 128-row x 64-column bf16 box (16 KB)
constexpr int TILE = 2 * HALF;     // one 128 x 128 bf16 tile (32 KB)
constexpr int STAGES = 2;
constexpr int NT = 16 * 128 * 2;   // a 16 x 128 bf16 operand tile (two 16 x 64 halves)
constexpr int OBOX = 32 * 64 * 2;  // one 32-token x 64-column output box (4 KB)
constexpr int SEG_BLOCKS = 8;      // blocks (1024 tokens) per segment when the sequence is split
constexpr int WIDE_HEADS = 96;     // from this many heads on (2/3 of 148 SMs): one segment per head
constexpr int W_CV = 4, W_FM = 12, FM_THREADS = 256, W_TMA = 20, W_MMA = 21, WARPS = 22, THREADS = WARPS * 32;
constexpr uint32_t T_ST = 0, T_OT = 128, T_P = 256, T_SA = 384, T_Z = 448, T_QZ = 464, TMEM_COLS = 512;
// stages | z operand tile | ones tile | 2 teams x staging (2 boxes) | 1/den | barriers
constexpr int OFF_ZB = STAGES * 3 * TILE, OFF_ONES = OFF_ZB + NT, OFF_STG = OFF_ONES + NT;
constexpr int OFF_INV = OFF_STG + 2 * 2 * OBOX, OFF_BAR = OFF_INV + TB * 4;
constexpr int SMEM = 1024 /*align*/ + OFF_BAR + 256;

__device__ int g_error = 0;  // set when a bounded wait expires

struct Params {
  float *ws;  // [B*H][G][D*D + D]: S^T (row d' holds S[:, d']) then z
  int H, T, G, blocks_per_seg, total_blocks, phase;
};

__device__ __forceinline__ bool wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return sm100::mbar_wait(bar, parity, abort_flag, &g_error);
}
// the same, with one outcome for the whole warp (warp-collective TMEM accesses follow)
__device__ __forceinline__ bool wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return __all_sync(0xffffffffu, wait(bar, parity, abort_flag));
}
// named barrier `id` over one team (128 threads); true iff `ok` held for all of them
__device__ __forceinline__ bool team_and(int id, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, 128, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void team_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// phi(x) = elu(x) + 1 = max(x, 0) + exp(min(x, 0)) on 8 bf16 values in place.
// max/min/add in bf16x2 are exact here (the add is x + 1 for x > 0 and 0 + e
// otherwise), so each result is the bf16 rounding of the fp32 value.
__device__ __forceinline__ void phi8(uint4 &v) {
  uint32_t *w = reinterpret_cast<uint32_t *>(&v);
  const __nv_bfloat162 zero = __float2bfloat162_rn(0.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162 *>(&w[i]);
    const float2 m = __bfloat1622float2(__hmin2(x, zero));
    const __nv_bfloat162 e = __floats2bfloat162_rn(__expf(m.x), __expf(m.y));
    const __nv_bfloat162 r = __hadd2(__hmax2(x, zero), e);
    w[i] = *reinterpret_cast<const uint32_t *>(&r);
  }
}

// byte offset of element (r, c) in a tile of 128-byte swizzled rows grouped
// in boxes of `rows` x 64 columns (the layout TMA uses with SWIZZLE_128B)
__device__ __forceinline__ uint32_t swz_off(int r, int c, int rows) {
  return (c >> 6) * (rows * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2;
}

// K-major operand (rows x 128, K = the 128 columns) in two 64-column boxes of
// `box_bytes`: K-step kk of 16 columns
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk, int box_bytes) {
  return smem_desc(base + (kk >> 2) * box_bytes + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (K = the 128 rows, MN = the 128 columns): K-step kk of 16 rows
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int kk) { return smem_desc(base + kk * 2048, HALF, 1024); }

__global__ void __launch_bounds__(THREADS, 1)
    linattn_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                      const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mo,
                      const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sZb = smem + OFF_ZB;      // [16 x 128] bf16: row 0 z_hi, row 1 z_lo, rest 0
  uint8_t *sOnes = smem + OFF_ONES;  // [16 x 128] bf16: row 0 ones, rest 0
  float *sInv = reinterpret_cast<float *>(smem + OFF_INV);  // [TB] 1 / denominator
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *full = bars, *empty = bars + 2, *fm_done = bars + 4;
  uint64_t *q_done = bars + 6, *s_full = bars + 7, *sa_ready = bars + 8, *p_ready = bars + 9, *o_full = bars + 10,
           *o_free = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x / p.G, seg = blockIdx.x % p.G;
  const int b = bh / p.H, h = bh % p.H;
  const bool out_pass = p.phase == 1;
  const bool seeded = out_pass && seg > 0;
  const int blk0 = seg * p.blocks_per_seg;
  const int nblk = min(p.blocks_per_seg, p.total_blocks - blk0);
  float *ws_seg = p.ws + ((int64_t)bh * p.G + seg) * (D * D + D);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&fm_done[s], FM_THREADS);
    }
    mbar_init(q_done, 1);
    mbar_init(s_full, 1);
    mbar_init(sa_ready, 256);
    mbar_init(p_ready, 128);
    mbar_init(o_full, 1);
    mbar_init(o_free, 256);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == W_TMA && lane == 0) {
    prefetch_map(&mq);
    prefetch_map(&mk);
    prefetch_map(&mv);
    prefetch_map(&mo);
  }
  // constant operand tiles: ones in row 0 of sOnes, zeros elsewhere (row 0 of
  // a swizzled tile is unpermuted)
  for (int i = threadIdx.x; i < 2 * NT / 16; i += THREADS) {
    const int tile = i / (NT / 16), o = (i % (NT / 16)) * 16;
    const bool ones = tile == 1 && (o % 2048) < 128;
    const uint32_t w = ones ? 0x3F803F80u : 0u;
    *reinterpret_cast<uint4 *>(smem + OFF_ZB + tile * NT + o) = make_uint4(w, w, w, w);
  }
  fence_proxy_async_smem();
  if (warp == W_MMA) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == W_TMA) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t bytes = (out_pass ? 3 : 2) * TILE;
      for (int c = 0; c < nblk; ++c) {
        const int st = c & 1;
        if (!wait(&empty[st], ((c >> 1) & 1) ^ 1, abort_flag)) break;
        uint8_t *slot = smem + st * 3 * TILE;
        const int t0 = (blk0 + c) * TB;
        mbar_expect_tx(&full[st], bytes);
        for (int j = 0; j < 2; ++j) {
          if (out_pass) tma_load_4d(slot + j * HALF, &mq, &full[st], j * 64, t0, h, b);
          tma_load_4d(slot + TILE + j * HALF, &mk, &full[st], j * 64, t0, h, b);
          tma_load_4d(slot + 2 * TILE + j * HALF, &mv, &full[st], j * 64, t0, h, b);
        }
      }
    }
  } else if (warp == W_MMA) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t ID_KK = idesc_bf16(128, 128, 0, 0), ID_MM = idesc_bf16(128, 128, 1, 1),
                         ID_MK = idesc_bf16(128, 128, 1, 0), ID_QZ = idesc_bf16(128, 16, 0, 0),
                         ID_Z = idesc_bf16(128, 16, 1, 0);
      const uint32_t zb = smem_u32(sZb), ones = smem_u32(sOnes);
      for (int c = 0; c < nblk; ++c) {
        const int st = c & 1;
        if (!wait(&fm_done[st], (c >> 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t q = smem_u32(smem + st * 3 * TILE), k = q + TILE, v = q + 2 * TILE;
        const bool update = !out_pass || c + 1 < nblk;
        if (out_pass) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_f16(tmem + T_P, desc_k(q, kk, HALF), desc_k(k, kk, HALF), ID_KK, kk > 0);
          if (!wait(sa_ready, c & 1, abort_flag)) break;
          if (c > 0 && !wait(o_free, (c - 1) & 1, abort_flag)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            umma_f16_ts(tmem + T_OT, tmem + T_SA + kk * 8, desc_k(q, kk, HALF), ID_KK, kk > 0);
            umma_f16(tmem + T_QZ, desc_k(q, kk, HALF), desc_k(zb, kk, NT / 2), ID_QZ, kk > 0);
          }
          umma_commit(q_done);
        }
        if (update) {
          const uint32_t acc0 = (out_pass || c > 0) ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            umma_f16(tmem + T_ST, desc_mn(v, kk), desc_mn(k, kk), ID_MM, acc0 | (kk > 0));
            umma_f16(tmem + T_Z, desc_mn(k, kk), desc_k(ones, kk, NT / 2), ID_Z, acc0 | (kk > 0));
          }
          if (out_pass || c + 1 == nblk) umma_commit(s_full);
        }
        if (out_pass) {
          if (!wait(p_ready, c & 1, abort_flag)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_f16(tmem + T_OT, desc_mn(v, kk), desc_k(q, kk, HALF), ID_MK, 1u);
          umma_commit(o_full);
        }
        umma_commit(&empty[st]);
      }
    }
  } else if (warp >= W_FM) {
    // ---------------- feature map (256 threads, in place, any element order) ----------------
    const int f = threadIdx.x - W_FM * 32;
    for (int c = 0; c < nblk; ++c) {
      const int st = c & 1;
      if (!wait(&full[st], (c >> 1) & 1, abort_flag)) break;
      uint8_t *slot = smem + st * 3 * TILE;
      for (int tile = out_pass ? 0 : 1; tile < 2; ++tile) {
        uint4 *base = reinterpret_cast<uint4 *>(slot + tile * TILE);
#pragma unroll 4
        for (int j = 0; j < TILE / 16 / FM_THREADS; ++j) {
          uint4 v = base[f + j * FM_THREADS];
          phi8(v);
          base[f + j * FM_THREADS] = v;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&fm_done[st]);
    }
  } else if (warp < W_CV) {
    // ---------------- score epilogue (rows t = 32*warp + lane) ----------------
    if (out_pass) {
      const int t = warp * 32 + lane;
      const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
      for (int c = 0; c < nblk; ++c) {
        const int st = c & 1;
        if (!wait_warp(q_done, c & 1, abort_flag)) break;
        tc_fence_after();
        uint8_t *pt = smem + st * 3 * TILE;  // P overwrites the consumed phi(Q) tile
        float rowsum = 0.f;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
          uint32_t packed[16];
          if (g > warp) {  // whole 32-column group above the diagonal
#pragma unroll
            for (int i = 0; i < 16; ++i) packed[i] = 0u;
          } else {
            uint32_t r[32];
            tmem_ld32(lane_base + T_P + g * 32, r);
            if (g == warp) {  // the diagonal group: s = 32g + j <= t  <=>  j <= lane
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j > lane) r[j] = 0u;
            }
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float a = __uint_as_float(r[j]), a1 = __uint_as_float(r[j + 1]);
              rowsum += a + a1;
              packed[j / 2] = pack_bf16(a, a1);
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4 *>(pt + swz_off(t, g * 32 + i * 8, TB)) =
                make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
        }
        uint32_t z0, z1;
        tmem_ld2(lane_base + T_QZ, z0, z1);
        sInv[t] = 1.f / (rowsum + (__uint_as_float(z0) + __uint_as_float(z1)));
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(p_ready);
      }
    }
  } else {
    // ------ state conversion and output epilogue: two teams, lanes d = 32*(warp%4) + lane ------
    const int team = (warp - W_CV) >> 2, quad = warp & 3, bar_id = 2 + team;
    const int d = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const bool leader = (warp & 3) == 0 && lane == 0;
    uint8_t *stg = smem + OFF_STG + team * 2 * OBOX;
    // z (fp32, TMEM lane d) -> bf16 hi/lo in rows 0 and 1 of the z operand tile
    auto publish_z = [&](float z) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(z);
      const __nv_bfloat16 lo = __float2bfloat16_rn(z - __bfloat162float(hi));
      *reinterpret_cast<__nv_bfloat16 *>(sZb + swz_off(0, d, 16)) = hi;
      *reinterpret_cast<__nv_bfloat16 *>(sZb + swz_off(1, d, 16)) = lo;
    };
    if (out_pass) {
      // seed S^T (fp32) and its bf16 copy (team 0: columns 0-63, team 1: 64-127) and z
#pragma unroll 1
      for (int g = team * 4; g < team * 4 + 4; ++g) {
        uint32_t w[16], hw[8];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = seeded ? __float_as_uint(ws_seg[(int64_t)d * D + g * 16 + i]) : 0u;
        tmem_st16(lane_base + T_ST + g * 16, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) hw[i] = pack_bf16(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
        tmem_st8(lane_base + T_SA + g * 8, hw);  // columns 16g..16g+15 as bf16 pairs
      }
      if (team == 0) {
        uint32_t w[16];
        const float z = seeded ? ws_seg[D * D + d] : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = i == 0 ? __float_as_uint(z) : 0u;
        tmem_st16(lane_base + T_Z, w);
        publish_z(z);
        fence_proxy_async_smem();
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(sa_ready);
      const bool odd = lane & 1;
      const int dcol = d & ~1;
      for (int c = 0; c < nblk; ++c) {
        if (c + 1 < nblk) {
          // S^T and z after this block -> operands of the next block
          if (!team_and(bar_id, wait_warp(s_full, c & 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll 1
          for (int g = team * 2; g < team * 2 + 2; ++g) {
            uint32_t r[32], hw[16];
            tmem_ld32(lane_base + T_ST + g * 32, r);
#pragma unroll
            for (int i = 0; i < 16; ++i) hw[i] = pack_bf16(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            tmem_st16(lane_base + T_SA + g * 16, hw);
          }
          if (team == 0) {
            publish_z(__uint_as_float(tmem_ld1(lane_base + T_Z)));
            fence_proxy_async_smem();
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(sa_ready);
        }
        // output rows 64*team .. 64*team+63 of this block: O^T and the
        // denominators are read into registers first, so the accumulator is
        // released before the (slower) staging and TMA stores
        if (!team_and(bar_id, wait_warp(o_full, c & 1, abort_flag) && wait_warp(p_ready, c & 1, abort_flag))) break;
        tc_fence_after();
        const int t0 = (blk0 + c) * TB;
        // tokens j and j+4 in one step: the even lane of a pair keeps token j,
        // the odd lane token j+4, each as the two adjacent columns dcol, dcol+1
        uint32_t w[2][16];
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          const int g = team * 2 + gi;
          uint32_t r[32];
          tmem_ld32(lane_base + T_OT + g * 32, r);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = (jj & 3) + (jj >> 2) * 8;
            const float a = __uint_as_float(r[j]) * sInv[g * 32 + j];
            const float a4 = __uint_as_float(r[j + 4]) * sInv[g * 32 + j + 4];
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? a : a4, 1);
            w[gi][jj] = odd ? pack_bf16(recv, a4) : pack_bf16(a, recv);
          }
        }
        tc_fence_before();
        mbar_arrive(o_free);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          if (leader) bulk_wait_read<0>();  // the previous store has read the staging buffer
          team_sync(bar_id);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = (jj & 3) + (jj >> 2) * 8;
            *reinterpret_cast<uint32_t *>(stg + swz_off(odd ? j + 4 : j, dcol, 32)) = w[gi][jj];
          }
          fence_proxy_async_smem();
          team_sync(bar_id);
          if (leader) {
            const int tok = t0 + (team * 2 + gi) * 32;
            tma_store_4d(&mo, stg, 0, tok, h, b);
            tma_store_4d(&mo, stg + OBOX, 64, tok, h, b);
            bulk_commit();
          }
        }
      }
      if (leader) bulk_wait<0>();
    } else if (wait_warp(s_full, 0, abort_flag)) {
      // state pass (s_full is committed once, after the last block): the
      // segment's S^T total (team 0: columns 0-63, team 1: 64-127) and z -> workspace
      tc_fence_after();
#pragma unroll 1
      for (int g = team * 2; g < team * 2 + 2; ++g) {
        uint32_t r[32];
        tmem_ld32(lane_base + T_ST + g * 32, r);
        float4 *dst = reinterpret_cast<float4 *>(ws_seg + (int64_t)d * D + g * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                               __uint_as_float(r[4 * i + 3]));
      }
      if (team == 0) ws_seg[D * D + d] = __uint_as_float(tmem_ld1(lane_base + T_Z));
    }
  }

  // teardown: every role has left its loop (normally or after an abort)
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && warp == W_TMA && lane == 0) {
    // bounded drain of copies that may still be landing in shared memory
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

// per head: segment states -> exclusive prefixes over the segments, in place
__global__ void __launch_bounds__(256) linattn_scan_kernel(float *ws, int G) {
  float *w = ws + (int64_t)blockIdx.x * G * (D * D + D);
  for (int i = threadIdx.x; i < D * D + D; i += blockDim.x) {
    float run = 0.f;
    for (int g = 0; g < G; ++g) {
      const float x = w[(int64_t)g * (D * D + D) + i];
      w[(int64_t)g * (D * D + D) + i] = run;
      run += x;
    }
  }
}

struct Operand {
  const void *ptr;
  int64_t sb, sh, ss;  // element strides of batch, head, token
};

// (d, t, h, b) tensor map with 64 x `rows` boxes; unit dims get a valid stride
static int make_map(CUtensorMap *m, const Operand &x, int64_t B, int64_t H, int64_t T, uint32_t rows) {
  const int64_t ss = x.ss;
  const int64_t sh = H > 1 ? x.sh : ss * T;
  const int64_t sb = B > 1 ? x.sb : sh * H;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)T, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)ss, (uint64_t)sh, (uint64_t)sb};
  const uint32_t box[4] = {64, rows, 1, 1};
  return make_bf16_map(m, x.ptr, 4, dims, strides, box);
}

// Segments per head: one, unless the heads alone cannot fill the GPU and the
// sequence is longer than one segment (the planner mirrors this rule).
int pick_segments(int BH, int T) {
  const int blocks = (T + TB - 1) / TB;
  if (blocks <= SEG_BLOCKS || BH >= WIDE_HEADS) return 1;
  return (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
}

size_t workspace_bytes(int BH, int G) { return (size_t)BH * G * (D * D + D) * sizeof(float); }

static int run(const Operand &q, const Operand &k, const Operand &v, const Operand &o, float *ws, int B, int H, int T,
               int G, cudaStream_t st, int device) {
  static ContextOnce attr;
  if (int s = attr.run(device, []() -> int {
        NKB_CUDA_TRY(cudaFuncSetAttribute(linattn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        return NKB_OK;
      }))
    return s;
  if (q.ss <= 0 || k.ss <= 0 || v.ss <= 0 || o.ss <= 0)
    return fail(NKB_ERR_UNSUPPORTED, "linattn: token strides must be positive");
  CUtensorMap mq, mk, mv, mo;
  if (int s = make_map(&mq, q, B, H, T, TB)) return s;
  if (int s = make_map(&mk, k, B, H, T, TB)) return s;
  if (int s = make_map(&mv, v, B, H, T, TB)) return s;
  if (int s = make_map(&mo, o, B, H, T, 32)) return s;
  Params p;
  p.ws = ws;
  p.H = H;
  p.T = T;
  p.G = G;
  p.total_blocks = (T + TB - 1) / TB;
  p.blocks_per_seg = G > 1 ? SEG_BLOCKS : p.total_blocks;
  const int BH = B * H;
  const unsigned grid = (unsigned)BH * (unsigned)G;
  if (G > 1) {
    p.phase = 0;
    linattn_tc_kernel<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, mo, p);
    if (int s = launch_status("linattn_tc_kernel(state)")) return s;
    linattn_scan_kernel<<<BH, 256, 0, st>>>(ws, G);
    if (int s = launch_status("linattn_scan_kernel")) return s;
  }
  p.phase = 1;
  linattn_tc_kernel<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, mo, p);
  return launch_status("linattn_tc_kernel(output)");
}

// "linattn": ptrs q k v o ws; ints B H T Dh G qb qh qs kb kh ks vb vh vs ob oh os
int check(const Step &s) {
  if (s.buf_ids.size() != 5 || s.ints.size() != 17) return fail(NKB_ERR_PLAN, "linattn: bad parameters");
  if (s.ints[3] != D) return fail(NKB_ERR_UNSUPPORTED, "linattn: head_dim must be 128");
  if (s.ints[2] % 64) return fail(NKB_ERR_UNSUPPORTED, "linattn: length must be a multiple of 64");
  if (s.ints[0] < 0 || s.ints[1] < 0 || s.ints[0] * s.ints[1] > (1 << 24) || s.ints[2] > (1 << 30))
    return fail(NKB_ERR_UNSUPPORTED, "linattn: sizes out of range");
  if (s.ints[4] != pick_segments((int)(s.ints[0] * s.ints[1]), (int)s.ints[2]))
    return fail(NKB_ERR_PLAN, "linattn: segment count does not match the kernel's segmentation");
  for (int i = 5; i < 17; ++i)
    if (s.ints[i] % 8 || s.ints[i] < 0) return fail(NKB_ERR_UNSUPPORTED, "linattn: strides must be multiples of 8");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  for (int i = 0; i < 4; ++i)
    if (reinterpret_cast<uintptr_t>(a.ptrs[i]) & 15) return fail(NKB_ERR_UNSUPPORTED, "linattn: unaligned base");
  const int B = (int)q[0], H = (int)q[1], T = (int)q[2], G = (int)q[4];
  if (B == 0 || H == 0 || T == 0) return NKB_OK;
  const Operand oq{a.ptrs[0], q[5], q[6], q[7]}, ok{a.ptrs[1], q[8], q[9], q[10]}, ov{a.ptrs[2], q[11], q[12], q[13]},
      oo{a.ptrs[3], q[14], q[15], q[16]};
  return run(oq, ok, ov, oo, static_cast<float *>(a.ptrs[4]), B, H, T, G, a.stream, a.device);
}

}  // namespace linattn

NKB_REGISTER_KERNEL("linattn", linattn::launch, linattn::check);

int linattn_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, linattn::g_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(linattn::g_error, &zero, sizeof(int)));
  return NKB_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant
// ---------------------------------------------------------------------------
// The planned path gets its segment-state workspace from the plan's scratch
// arena, which the runtime allocates when the plan is loaded.  Some callers
// cannot allocate device memory at the point where they run this kernel: a
// host process that has handed the whole GPU to its own caching allocator up
// front, or a latency-critical loop in which a cudaMalloc/cudaFree could
// block or synchronise the device.  For them the workspace lives in a fixed,
// file-scope device array of NKB_LINATTN_SCRATCH_BYTES: every GPU that loads
// this library holds it until the process exits, and every call shares it.
namespace linattn {

static __device__ __align__(256) unsigned char g_scratch[NKB_LINATTN_SCRATCH_BYTES];

static void *g_scratch_addr[64];
static unsigned long long g_scratch_ctx[64];
static std::mutex g_scratch_mu;

// Device address of the fixed workspace on the current device.  In host code
// `g_scratch` only names a host-side stand-in, so the address is looked up
// once per device with that device current -- and looked up again when the
// device's CUDA context changed (after a cudaDeviceReset the module, and the
// array with it, is loaded afresh at another address).
static int scratch_address(int device, void **out) {
  if (device < 0 || device >= 64) return fail(NKB_ERR_INVALID, "device index out of range");
  const unsigned long long ctx = context_id();
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[device] || ctx == 0 || g_scratch_ctx[device] != ctx) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(NKB_ERR_CUDA, std::string("cudaGetSymbolAddress(linear-attention scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[device] = ptr;
    g_scratch_ctx[device] = ctx;
  }
  *out = g_scratch_addr[device];
  return NKB_OK;
}

}  // namespace linattn
}  // namespace nkb

extern "C" int nkb_linear_attention_noalloc(const void *q, const void *k, const void *v, void *out, int64_t B,
                                            int64_t H, int64_t T, int64_t D, void *stream) {
  using namespace nkb;
  using namespace nkb::linattn;
  if (!q || !k || !v || !out) return fail(NKB_ERR_INVALID, "linear attention: NULL pointer");
  if (D != linattn::D) return fail(NKB_ERR_UNSUPPORTED, "linear attention: head_dim must be 128");
  if (B < 0 || H < 0 || T < 0 || T % 64) return fail(NKB_ERR_UNSUPPORTED, "linear attention: length must be a multiple of 64");
  // each factor bounded before the product is formed (caller-supplied sizes)
  if (B > (1 << 24) || H > (1 << 24) || B * H > (1 << 24) || T > (1 << 30))
    return fail(NKB_ERR_INVALID, "linear attention: sizes too large");
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  if (al & 15) return fail(NKB_ERR_UNSUPPORTED, "linear attention: pointers must be 16-byte aligned");
  if (B == 0 || H == 0 || T == 0) return NKB_OK;
  int dev = 0;
  NKB_CUDA_TRY(cudaGetDevice(&dev));
  const int BH = (int)(B * H);
  const int G = pick_segments(BH, (int)T);
  const size_t need = G > 1 ? workspace_bytes(BH, G) : 0;
  if (need > (size_t)NKB_LINATTN_SCRATCH_BYTES)
    return fail(NKB_ERR_INVALID, "linear attention: " + std::to_string(B) + "x" + std::to_string(H) +
                                     " heads need " + std::to_string(need) + " bytes of workspace, more than the fixed " +
                                     std::to_string((size_t)NKB_LINATTN_SCRATCH_BYTES) + " bytes of the allocation-free entry point");
  void *ws = nullptr;
  if (int s = scratch_address(dev, &ws)) return s;
  const int64_t sb = H * T * D, sh = T * D, ss = D;
  const Operand oq{q, sb, sh, ss}, ok{k, sb, sh, ss}, ov{v, sb, sh, ss}, oo{out, sb, sh, ss};
  return run(oq, ok, ov, oo, static_cast<float *>(ws), (int)B, (int)H, (int)T, G, static_cast<cudaStream_t>(stream), dev);
}
