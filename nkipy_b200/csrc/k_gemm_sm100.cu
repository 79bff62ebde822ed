// bf16 GEMM on the 5th-generation tensor cores (sm_100a): the HLO ``dot`` of
// NKIPy's matmul (reference core/ops/linalg.py:15-125) for bf16 operands with
// fp32 accumulation.
//
// Structure (one CTA per SM, persistent over output tiles of 128 x 256):
//   warp 0      TMA producer: 128B-swizzled A (128 x 64) and B (64 x 256)
//               tiles into a 4-stage shared-memory ring (mbarrier complete_tx);
//   warp 1      allocates 512 TMEM columns, then one lane issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) and
//               tcgen05.commit to release smem stages / publish accumulators;
//   warps 2..5  epilogue: tcgen05.ld 32x32b.x32 of their TMEM lane quadrant,
//               fp32 -> bf16/fp32, 16-byte stores.
// Two TMEM accumulators (2 x 256 columns) let the epilogue of tile i overlap
// the main loop of tile i+1.  No cluster multicast is used anywhere: each CTA
// fetches its own tiles and L2 provides the reuse, so the same kernel is safe
// on multi-GPU runs.
//
// Fused all-reduce (row-parallel GEMMs under tensor parallelism): C is this
// rank's copy of a symmetric region; tiles are taken row block by row block,
// and after the epilogue stores a tile one thread adds 1 to that row block's
// arrival count on every rank (multimem.red through the multicast object).
// Four more warps per CTA (warps 6-9) reduce, as soon as a row block's count
// shows every rank's tiles, this CTA's share of this rank's part of the block
// (multimem.ld_reduce with fp32 accumulation, optionally + a residual, then
// multimem.st to every rank), while later tiles are still computing.  The last
// CTA of a rank clears the arrival counts and adds 1 to a done count on every
// rank, then waits until every rank is done.  Every wait is bounded.
//
// A may be K-major (row-major M x K) or M-major (stored K x M); B may be
// N-major (row-major K x N) or K-major (stored N x K).  Tensor maps are 3-D
// (inner, outer, batch).  Every mbarrier wait is bounded by a clock budget;
// on expiry the CTA raises a device error flag, stops issuing work, waits
// (bounded) for its in-flight copies, frees its TMEM and exits.

#include <cstdlib>

#include "sm100.cuh"

namespace nkb {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 1024 /*barriers*/ + 1024 /*align*/;
constexpr int TMEM_COLS = 512;
constexpr int THREADS = 192;

__device__ int g_device_error = 0;  // set when a bounded wait expires

struct Args {
  void *C;
  int64_t M, N, K, ldc, sC, batch;
  int c_f32, a_mn_major, b_k_major;
  int a_bcast, b_bcast;  // batch stride 0: every batch reads operand batch 0
  int tiles_m, tiles_n;
  int tiles_m2;  // 256-row tiles (CTA pairs)
  // epi == 1 (SwiGLU): B holds [gate | up] halves of width n_half; a CTA
  // computes 128 gate + the matching 128 up columns and writes
  // silu(gate) * up (N = n_half output columns).
  int epi;
  int64_t n_half;
  // epi == 2 (residual): C = bf16(bf16(A @ B) + R), R bf16 with row stride ldr
  const __nv_bfloat16 *res;
  int64_t ldr;
  // epi == 3 (rotary embedding): columns [rope_r0[i], rope_r1[i]) are heads of
  // rope_hd columns rotated in place; position = row % rope_seq; cos/sin are
  // bf16 tables [rope_seq][rope_hd / 2]
  const __nv_bfloat16 *rope_cos, *rope_sin;
  int64_t rope_r0[2], rope_r1[2];
  int rope_hd, rope_seq;
  // fused all-reduce (gemm_bf16_tcgen05<true>): C dense bf16 with N columns
  uint64_t ar_mc;               // C through the multicast object
  uint32_t *ar_flags;           // this rank's flag slot
  uint64_t ar_mc_flags;         // the slot through the multicast object
  const __nv_bfloat16 *ar_res;  // optional residual (dense, N columns): C = res + sum
  int ar_rank, ar_world;
  long long ar_wait;            // budget of each wait on the counts (SM clock cycles)
  // split-K (few output tiles, long K: the decode projections): work unit =
  // (tile, split); split s takes k-blocks [s * kb / ksplit, (s + 1) * kb / ksplit)
  // and stores its fp32 partial rows to ws[s][M][N]; a second kernel sums them
  int ksplit;
  float *ws;
  // raster: row tiles per group (a wave of CTAs walks the columns of one
  // group, sharing its A panels and each B column panel in L2)
  int group;
};

constexpr int AR_WARPS = 4, AR_T = AR_WARPS * 32;  // all-reduce warps per CTA
constexpr int AR_RUN = 64;                         // most row blocks reduced in one pass
constexpr int AR_THREADS = 192 + AR_T;

using namespace sm100;

// Bounded wait reporting into this kernel's device error flag.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  return sm100::mbar_wait(bar, parity, abort_flag, &g_device_error);
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Instruction descriptor: D fp32, A/B bf16, M=128, N=256.
__host__ __device__ constexpr uint32_t make_idesc(int a_mn_major, int b_mn_major) {
  return idesc_bf16(BM, BN, a_mn_major, b_mn_major);
}

// Tile t -> (row tile, column tile, batch); row tiles are 128 rows, or 256
// for a CTA pair (PAIR).
template <bool AR, bool PAIR>
__device__ __forceinline__ void tile_coords(int t, const Args &a, int &bm, int &bn, int &bb) {
  if (AR) {  // row block by row block, so blocks complete (and are reduced) in order
    bb = 0;
    bm = t / a.tiles_n;
    bn = t - bm * a.tiles_n;
    return;
  }
  const int tm = PAIR ? a.tiles_m2 : a.tiles_m;
  const int per_batch = tm * a.tiles_n;
  bb = t / per_batch;
  int r = t - bb * per_batch;
  const int group = a.group;
  const int group_span = group * a.tiles_n;
  const int g = r / group_span;
  const int first_m = g * group;
  const int gsize = min(tm - first_m, group);
  const int within = r - g * group_span;
  bm = first_m + within % gsize;
  bn = within / gsize;
}

// Work unit t -> tile coordinates and its range of k-blocks.
template <bool AR, bool PAIR>
__device__ __forceinline__ void unit_coords(int t, const Args &a, int k_blocks, int &bm, int &bn, int &bb, int &split,
                                            int &kb0, int &kb1) {
  split = 0;
  if (!AR && a.ksplit > 1) {
    const int per_split = a.tiles_m * a.tiles_n * (int)a.batch;
    split = t / per_split;
    t -= split * per_split;
  }
  tile_coords<AR, PAIR>(t, a, bm, bn, bb);
  const int ks = AR ? 1 : max(1, a.ksplit);
  kb0 = (int)((int64_t)split * k_blocks / ks);
  kb1 = (int)((int64_t)(split + 1) * k_blocks / ks);
}

// ---- fused all-reduce helpers ------------------------------------------------

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// +v on every rank's copy of a multicast address, ordered after this thread's
// (and, through a preceding barrier, its CTA's) earlier writes
__device__ __forceinline__ void mc_red_add_release(uint64_t addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
// sum over all ranks of 16 bytes of bf16 pairs at a multicast address (fp32
// accumulation inside the switch, one bf16 rounding)
__device__ __forceinline__ void mc_ld_reduce_bf16(uint64_t addr, uint32_t *r) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(addr)
               : "memory");
}
__device__ __forceinline__ void mc_st16(uint64_t addr, const uint32_t *r) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// barrier over `threads` threads that returns the AND of `pred` (uniform exits)
__device__ __forceinline__ bool named_bar_and(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Vectors (16 bytes) [lo, hi) of row block cc that this CTA reduces on this rank.
__device__ __forceinline__ void ar_piece(const Args &a, int cc, int64_t &lo, int64_t &hi) {
  const int64_t row_vecs = a.N / 8;
  const int64_t r0 = (int64_t)cc * BM;
  const int64_t nv = min((int64_t)BM, a.M - r0) * row_vecs;
  const int64_t rlo = nv * a.ar_rank / a.ar_world, rn = nv * (a.ar_rank + 1) / a.ar_world - rlo;
  lo = r0 * row_vecs + rlo + rn * blockIdx.x / gridDim.x;
  hi = r0 * row_vecs + rlo + rn * (blockIdx.x + 1) / gridDim.x;
}

// Warps 6.. of the fused kernel (AR_T threads, ct = 0..AR_T-1).
__device__ void ar_comm(const Args &a, int ct, volatile int *abort_flag) {
  const int lane = ct % 32;
  uint32_t *const cnt = a.ar_flags + SYMM_AR_CHUNKS;  // this rank's finished CTAs
  uint32_t *const done = cnt + 1;                     // finished ranks (every rank adds 1)
  const uint64_t mc_done = a.ar_mc_flags + 4ull * (SYMM_AR_CHUNKS + 1);
  // done counts of earlier launches: no rank can finish this launch before this
  // CTA has stored its tiles, which it does after this read
  const uint32_t d0 = ld_acquire_sys(done);
  const uint32_t need = (uint32_t)(a.tiles_n * a.ar_world);
  auto ready = [&](int cc) { return (int)(ld_acquire_sys(a.ar_flags + cc) - need) >= 0; };
  bool ok = true;
  int c = 0;
  while (c < a.tiles_m) {
    // warp-uniform: wait for row block c, then take the run of ready blocks after it (at most
    // AR_RUN: one block gives a thread less than one vector at 8 ranks, so a run of many blocks
    // is what keeps eight reductions in flight per thread)
    int ce = c;
    if (lane == 0) {
      ok = wait_counter_geq(a.ar_flags + c, need, a.ar_wait, abort_flag, 256);
      if (ok)
        for (ce = c + 1; ce < a.tiles_m && ce < c + AR_RUN && ready(ce);) ++ce;
    }
    ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
    ce = __shfl_sync(0xffffffffu, ce, 0);
    if (!ok) break;
    // this thread's vectors of blocks [c, ce), eight reductions in flight at a time
    int cc = c;
    int64_t lo, hi;
    ar_piece(a, cc, lo, hi);
    int64_t v = lo + ct;
    while (true) {
      int64_t addr[8];
      bool valid[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        while (v >= hi && cc + 1 < ce) {
          ++cc;
          ar_piece(a, cc, lo, hi);
          v = lo + ct;
        }
        valid[i] = v < hi;
        addr[i] = v;
        if (valid[i]) v += AR_T;
      }
      if (!valid[0]) break;
      uint32_t r[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (valid[i]) mc_ld_reduce_bf16(a.ar_mc + 16ull * addr[i], r[i]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (!valid[i]) continue;
        if (a.ar_res) {
          // the traced add after the all-reduce: bf16 + bf16, rounded once
          const uint4 x = *reinterpret_cast<const uint4 *>(a.ar_res + 8 * addr[i]);
          const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r[i][j]));
            const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&xw[j]));
            r[i][j] = pack_bf16(p.x + q.x, p.y + q.y);
          }
        }
        mc_st16(a.ar_mc + 16ull * addr[i], r[i]);
      }
    }
    __syncwarp();
    c = ce;
  }
  if (!ok) {
    atomicExch(&g_device_error, 1);
    *abort_flag = 1;
  }
  named_bar(2, AR_T);  // every all-reduce warp is past its last store
  if (ct == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const uint32_t prev = atomicAdd(cnt, 1u);
    if (prev == gridDim.x - 1) {
      // last CTA of this rank: every CTA has read its counts; clear them for the
      // next launch before telling the other ranks (whose next launch starts
      // only after they see every rank done)
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      *cnt = 0;
      for (int i = 0; i < a.tiles_m; ++i) a.ar_flags[i] = 0;
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      mc_red_add_release(mc_done, 1);
      const uint32_t target = d0 - d0 % (uint32_t)a.ar_world + (uint32_t)a.ar_world;
      if (!wait_counter_geq(done, target, a.ar_wait, nullptr, 256)) atomicExch(&g_device_error, 1);
    }
  }
}

// PAIR: a cluster of two CTAs computes 256 x 256 tiles with
// tcgen05.mma.cta_group::2 (M = 256): each CTA loads its own 128 rows of A
// and its own 128 columns of B (plain TMA loads, no multicast) and keeps its
// 128 rows of the accumulator in its own TMEM.  Both CTAs' loads complete on
// the leader's (rank 0) stage barriers; the leader's single MMA thread issues
// the products and signals stage release and accumulator completion to both
// CTAs (tcgen05.commit multicast); both epilogues report a drained
// accumulator to the leader.  Per SM this moves 32 KB through shared memory
// per 64-deep k-block instead of 48 KB for the same flops.
template <bool AR, bool PAIR>
__global__ void __launch_bounds__(AR ? AR_THREADS : THREADS, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Args args) {
  constexpr int NST = PAIR ? 6 : STAGES;                             // stages of the load ring
  constexpr int B_BYTES = PAIR ? (BN / 2) * BK * 2 : B_STAGE_BYTES;  // this CTA's B per stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + NST * A_STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + NST * B_BYTES);
  uint64_t *full = bars;                  // [NST]
  uint64_t *empty = bars + NST;           // [NST]
  uint64_t *acc_full = bars + 2 * NST;      // [2]
  uint64_t *acc_empty = bars + 2 * NST + 2;  // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * NST + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = PAIR ? cluster_rank() : 0;  // 0: the leader of the pair
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // first tile of this CTA (pair)
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int num_tiles =
      (PAIR ? args.tiles_m2 : args.tiles_m) * args.tiles_n * (int)args.batch * (AR ? 1 : max(1, args.ksplit));
  const int k_blocks = (int)((args.K + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      // drained by the 128 epilogue threads, or by the 4 + 4 epilogue warps of a pair
      mbar_init(&acc_empty[i], PAIR ? 8 : 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&map_a);
    prefetch_map(&map_b);
  }
  if (warp == 1) {
    if (PAIR)
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
    else
      tmem_alloc(tmem_slot, TMEM_COLS);
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // the leader's barriers exist before the peer signals them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the leader's stage and accumulator-drained barriers, as seen from this CTA
  const uint32_t full_leader = PAIR ? map_to_rank(smem_u32(full), 0) : 0;
  const uint32_t acc_empty_leader = PAIR ? map_to_rank(smem_u32(acc_empty), 0) : 0;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = unit0; t < num_tiles && ok; t += units) {
        int bm, bn, bb, split, kb0, kb1;
        unit_coords<AR, PAIR>(t, args, k_blocks, bm, bn, bb, split, kb0, kb1);
        if (PAIR) {
          const int row0 = (bm * 2 + (int)rank) * BM;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % NST;
            const uint32_t ph = (it / NST) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            // the leader expects both CTAs' bytes; the peer's may land first
            if (rank == 0) mbar_expect_tx(&full[s], 2 * (A_STAGE_BYTES + B_BYTES));
            const uint32_t fb = full_leader + 8u * s;
            uint8_t *a_dst = sA + s * A_STAGE_BYTES;
            uint8_t *b_dst = sB + s * B_BYTES;
            if (!args.a_mn_major) {
              tma_load_3d_pair(a_dst, &map_a, fb, kb * BK, row0, args.a_bcast ? 0 : bb);
            } else {
              for (int j = 0; j < BM / 64; ++j)
                tma_load_3d_pair(a_dst + j * (64 * BK * 2), &map_a, fb, row0 + j * 64, kb * BK, args.a_bcast ? 0 : bb);
            }
            if (args.b_k_major) {
              tma_load_3d_pair(b_dst, &map_b, fb, kb * BK, bn * BN + (int)rank * (BN / 2), args.b_bcast ? 0 : bb);
            } else {
              // SwiGLU: the leader holds the 128 gate columns, the peer the matching 128 up columns
              const int c0 = args.epi == 1 ? (int)rank * (int)args.n_half + bn * (BN / 2) : bn * BN + (int)rank * (BN / 2);
              for (int j = 0; j < BN / 128; ++j)
                tma_load_3d_pair(b_dst + j * (64 * BK * 2), &map_b, fb, c0 + j * 64, kb * BK, args.b_bcast ? 0 : bb);
            }
          }
          continue;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], A_STAGE_BYTES + B_STAGE_BYTES);
          uint8_t *a_dst = sA + s * A_STAGE_BYTES;
          uint8_t *b_dst = sB + s * B_STAGE_BYTES;
          if (!args.a_mn_major) {
            tma_load_3d(a_dst, &map_a, &full[s], kb * BK, bm * BM, args.a_bcast ? 0 : bb);
          } else {
            for (int j = 0; j < BM / 64; ++j)
              tma_load_3d(a_dst + j * (64 * BK * 2), &map_a, &full[s], bm * BM + j * 64, kb * BK, args.a_bcast ? 0 : bb);
          }
          if (args.b_k_major) {
            tma_load_3d(b_dst, &map_b, &full[s], kb * BK, bn * BN, args.b_bcast ? 0 : bb);
          } else if (args.epi == 1) {
            const int n0 = bn * (BN / 2);
            for (int j = 0; j < BN / 64; ++j) {
              const int col = (j < 2) ? n0 + j * 64 : (int)args.n_half + n0 + (j - 2) * 64;
              tma_load_3d(b_dst + j * (64 * BK * 2), &map_b, &full[s], col, kb * BK, args.b_bcast ? 0 : bb);
            }
          } else {
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(b_dst + j * (64 * BK * 2), &map_b, &full[s], bn * BN + j * 64, kb * BK, args.b_bcast ? 0 : bb);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (PAIR && lane == 0 && rank == 0) {
      // the leader issues the pair's products: M = 256 (128 rows in each CTA), N = 256
      const uint32_t idesc = idesc_bf16(2 * BM, BN, args.a_mn_major, args.b_k_major ? 0 : 1);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = unit0; t < num_tiles && ok; t += units, ++local) {
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int bm, bn, bb, split, kb0, kb1;
        unit_coords<AR, PAIR>(t, args, k_blocks, bm, bn, bb, split, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NST;
          const uint32_t ph = (it / NST) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = args.a_mn_major ? smem_desc(a_addr + k * 2048, 64 * BK * 2, 1024)
                                                : smem_desc(a_addr + k * 32, 16, 1024);
            const uint64_t db = args.b_k_major ? smem_desc(b_addr + k * 32, 16, 1024)
                                               : smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024);
            umma_f16_pair(d_tmem, da, db, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[s]);  // stage s free in both CTAs once these MMAs have read it
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[acc]);  // both CTAs' accumulator rows ready
      }
    } else if (!PAIR && lane == 0) {
      const uint32_t idesc = make_idesc(args.a_mn_major, args.b_k_major ? 0 : 1);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int bm, bn, bb, split, kb0, kb1;
        unit_coords<AR, PAIR>(t, args, k_blocks, bm, bn, bb, split, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 16 elements = 32 bytes inside the 128B swizzle row;
            // MN-major: advance 16 K-rows = 2048 bytes.
            const uint64_t da = args.a_mn_major ? smem_desc(a_addr + k * 2048, 64 * BK * 2, 1024)
                                                : smem_desc(a_addr + k * 32, 16, 1024);
            const uint64_t db = args.b_k_major ? smem_desc(b_addr + k * 32, 16, 1024)
                                               : smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024);
            umma_f16(d_tmem, da, db, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // stage s free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);  // accumulator ready for the epilogue
      }
    }
  } else if (AR && warp >= 6) {
    // ---------------- all-reduce (warps 6..) ----------------
    ar_comm(args, threadIdx.x - 192, abort_flag);
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp % 4;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    // the accumulator has been read: every thread (one CTA), or each warp once (pair, at the leader)
    auto drained = [&](int acc) {
      tc_fence_before();
      if (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader + 8u * acc);
      } else {
        mbar_arrive(&acc_empty[acc]);
      }
    };
    int local = 0;
    for (int t = unit0; t < num_tiles; t += units, ++local) {
      int bm, bn, bb, split, kb0, kb1;
      unit_coords<AR, PAIR>(t, args, k_blocks, bm, bn, bb, split, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      bool got = mbar_wait(&acc_full[acc], acc_ph, abort_flag);
      if (AR) got = named_bar_and(1, 128, got);  // the four warps leave together
      if (!got) break;
      tc_fence_after();
      const int bm_own = PAIR ? bm * 2 + (int)rank : bm;  // this CTA's 128-row block
      const int64_t row = (int64_t)bm_own * BM + row_in_tile;
      const bool row_ok = row < args.M;
      if (args.epi == 1) {
        const int64_t col0 = (int64_t)bn * (BN / 2);
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, g);
          tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + BN / 2 + c * 32, u);
          const int64_t col = col0 + c * 32;
          if (!row_ok || col >= args.N) continue;
          __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(args.C) + bb * args.sC + row * args.ldc + col;
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float o2[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              // silu(g) * u with the traced bf16 node sequence:
              // negate, exponential, 1 + ., 1 / ., g * ., . * u (each rounded)
              const float gv = bf16r(__uint_as_float(g[j + t]));
              const float uv = bf16r(__uint_as_float(u[j + t]));
              const float e = bf16r(expf(-gv));
              const float d = bf16r(1.0f + e);
              const float r = bf16r(1.0f / d);
              const float sg = bf16r(gv * r);
              o2[t] = sg * uv;
            }
            __nv_bfloat162 h = __floats2bfloat162_rn(o2[0], o2[1]);
            packed[j / 2] = *reinterpret_cast<uint32_t *>(&h);
          }
          if (col + 32 <= args.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<uint4 *>(dst + 2 * j) = make_uint4(packed[j], packed[j + 1], packed[j + 2], packed[j + 3]);
          } else {
            for (int j = 0; j < 32 && col + j < args.N; ++j)
              dst[j] = reinterpret_cast<__nv_bfloat16 *>(packed)[j];
          }
        }
        drained(acc);
        continue;
      }
      const int64_t col0 = (int64_t)bn * BN;
      if (args.epi == 3) {
        // the traced rotation of rope.py:34-57 on bf16 values, each node rounded:
        //   lo = x0 * cos - x1 * sin,  hi = x0 * sin + x1 * cos  (x0 = column d, x1 = d + hd/2)
        const int hd = args.rope_hd, half = hd / 2;
        const int64_t pos = row % args.rope_seq;
        const uint32_t lane_acc = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
        for (int c = 0; c < BN / 32; ++c) {
          const int64_t col = col0 + c * 32;
          int rr = -1;
          for (int i = 0; i < 2; ++i)
            if (col >= args.rope_r0[i] && col < args.rope_r1[i]) rr = i;
          const int d = rr < 0 ? 0 : (int)((col - args.rope_r0[rr]) % hd);
          if (rr >= 0 && d >= half) continue;  // written together with its partner chunk
          uint32_t x0[32], x1[32];
          tmem_ld32(lane_acc + c * 32, x0);
          if (rr >= 0) tmem_ld32(lane_acc + (c + half / 32) * 32, x1);
          if (!row_ok || col >= args.N) continue;
          __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(args.C) + bb * args.sC + row * args.ldc + col;
          uint32_t lo[16], hi[16];
          if (rr < 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) lo[j] = pack_bf16(__uint_as_float(x0[2 * j]), __uint_as_float(x0[2 * j + 1]));
          } else {
            // the 32 cos / sin values of this row's position, 16 bytes at a time (the
            // planner passes 16-byte aligned tables and d is a multiple of 32)
            const uint4 *cs4 = reinterpret_cast<const uint4 *>(args.rope_cos + pos * half + d);
            const uint4 *sn4 = reinterpret_cast<const uint4 *>(args.rope_sin + pos * half + d);
            uint4 cv[4], sv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              cv[q] = cs4[q];
              sv[q] = sn4[q];
            }
            const __nv_bfloat16 *cs = reinterpret_cast<const __nv_bfloat16 *>(cv);
            const __nv_bfloat16 *sn = reinterpret_cast<const __nv_bfloat16 *>(sv);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float l2[2], h2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float a = bf16r(__uint_as_float(x0[j + e])), b = bf16r(__uint_as_float(x1[j + e]));
                const float co = __bfloat162float(cs[j + e]), si = __bfloat162float(sn[j + e]);
                l2[e] = bf16r(bf16r(a * co) - bf16r(b * si));
                h2[e] = bf16r(a * si) + bf16r(b * co);
              }
              lo[j / 2] = pack_bf16(l2[0], l2[1]);
              hi[j / 2] = pack_bf16(h2[0], h2[1]);
            }
          }
          const bool vec = col + 32 <= args.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            if (w == 1 && rr < 0) break;
            const uint32_t *src = w ? hi : lo;
            __nv_bfloat16 *o = dst + w * half;
            if (vec) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4 *>(o + 2 * j) = make_uint4(src[j], src[j + 1], src[j + 2], src[j + 3]);
            } else {
              for (int j = 0; j < 32 && col + w * half + j < args.N; ++j) o[j] = reinterpret_cast<const __nv_bfloat16 *>(src)[j];
            }
          }
        }
        drained(acc);
        continue;
      }
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
        const int64_t col = col0 + c * 32;
        if (!row_ok || col >= args.N) continue;
        const bool full_chunk = col + 32 <= args.N;
        if (!AR && args.ksplit > 1) {
          // this split's fp32 partial of the row (summed and rounded by splitk_reduce)
          float *dst = args.ws + ((int64_t)split * args.M + row) * args.N + col;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<uint4 *>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          } else {
            for (int j = 0; j < 32 && col + j < args.N; ++j) dst[j] = __uint_as_float(r[j]);
          }
          continue;
        }
        if (args.c_f32) {
          float *dst = static_cast<float *>(args.C) + bb * args.sC + row * args.ldc + col;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<uint4 *>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          } else {
            for (int j = 0; j < 32 && col + j < args.N; ++j) dst[j] = __uint_as_float(r[j]);
          }
        } else {
          __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(args.C) + bb * args.sC + row * args.ldc + col;
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            packed[j] = *reinterpret_cast<uint32_t *>(&h);
          }
          if (args.epi == 2) {
            // the traced add after the product: both operands bf16, the sum rounded once more
            const __nv_bfloat16 *src = args.res + row * args.ldr + col;
            if (full_chunk && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const uint4 rv = *reinterpret_cast<const uint4 *>(src + 2 * j);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&packed[j + i]));
                  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&rw[i]));
                  packed[j + i] = pack_bf16(a.x + b.x, a.y + b.y);
                }
              }
            } else {
              for (int j = 0; j < 32 && col + j < args.N; ++j) {
                const float a = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(packed)[j]);
                reinterpret_cast<__nv_bfloat16 *>(packed)[j] = __float2bfloat16_rn(a + __bfloat162float(src[j]));
              }
            }
          }
          if (full_chunk && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<uint4 *>(dst + 2 * j) = make_uint4(packed[j], packed[j + 1], packed[j + 2], packed[j + 3]);
          } else {
            for (int j = 0; j < 32 && col + j < args.N; ++j) dst[j] = reinterpret_cast<const __nv_bfloat16 *>(packed)[j];
          }
        }
      }
      drained(acc);
      if (AR) {
        named_bar(1, 128);  // the tile is stored by all four warps
        if (warp == 2 && lane == 0) {
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          mc_red_add_release(args.ar_mc_flags + 4ull * bm_own, 1);
        }
      }
    }
  }

  // teardown: every role has left its loop (normally or after an abort)
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // neither CTA of the pair still signals the other's barriers
  else
    __syncthreads();
  if (*abort_flag && warp == 0 && lane == 0) {
    // bounded drain of copies that may still be landing in shared memory
    const long long t0 = clock64();
    while (clock64() - t0 < 2000000) {
    }
  }
  if (PAIR)
    cluster_sync();
  else
    __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int make_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t batch,
                    uint64_t outer_stride_elems, uint64_t batch_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  const uint64_t dims[3] = {inner, outer, batch};
  const uint64_t strides[2] = {outer_stride_elems, batch > 1 ? batch_stride_elems : outer * outer_stride_elems};
  const uint32_t box[3] = {box_inner, box_outer, 1};
  return make_bf16_map(map, base, 3, dims, strides, box);
}

// Can the tcgen05 path take these operands?  (16-byte aligned bases and
// strides, as TMA requires; batch strides of broadcast operands are 0.)
bool tc_eligible(const void *A, const void *B, int64_t lda, int64_t ldb, int64_t sA, int64_t sB, int64_t batch) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(A) || !al(B)) return false;
  if (lda % 8 || ldb % 8) return false;
  if (batch > 1 && ((sA % 8) || (sB % 8))) return false;
  return true;
}

// C = bf16(sum over s of ws[s]) for the split-K partials ws[ksplit][M][N] (fp32).
template <bool VEC>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float *__restrict__ ws, __nv_bfloat16 *__restrict__ C,
                                                            int64_t M, int64_t N, int64_t ldc, int ks) {
  pdl_wait();
  pdl_trigger();
  const int64_t per = VEC ? 4 : 1;
  const int64_t n = M * N / per;
  const int64_t plane = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * per, row = e / N, col = e - row * N;
    if (VEC) {
      // up to kFlight partials loaded before the first add (one round trip),
      // then summed in split order
      constexpr int kFlight = 16;
      float4 acc = *reinterpret_cast<const float4 *>(ws + e);
      float4 v[kFlight - 1];
#pragma unroll
      for (int s = 1; s < kFlight; ++s)
        if (s < ks) v[s - 1] = *reinterpret_cast<const float4 *>(ws + s * plane + e);
#pragma unroll
      for (int s = 1; s < kFlight; ++s)
        if (s < ks) {
          acc.x += v[s - 1].x;
          acc.y += v[s - 1].y;
          acc.z += v[s - 1].z;
          acc.w += v[s - 1].w;
        }
      for (int s = kFlight; s < ks; ++s) {
        const float4 u = *reinterpret_cast<const float4 *>(ws + s * plane + e);
        acc.x += u.x;
        acc.y += u.y;
        acc.z += u.z;
        acc.w += u.w;
      }
      __nv_bfloat16 *dst = C + row * ldc + col;
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t *>(&lo);
      u.y = *reinterpret_cast<const uint32_t *>(&hi);
      *reinterpret_cast<uint2 *>(dst) = u;
    } else {
      float acc = ws[e];
#pragma unroll 8
      for (int s = 1; s < ks; ++s) acc += ws[s * plane + e];
      C[row * ldc + col] = __float2bfloat16_rn(acc);
    }
  }
}

int splitk_reduce(const float *ws, __nv_bfloat16 *C, int64_t M, int64_t N, int64_t ldc, int ks, cudaStream_t st,
                  int device) {
  const bool vec = N % 4 == 0 && ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(C) & 7) == 0;
  const int64_t work = M * N / (vec ? 4 : 1);
  const unsigned grid = (unsigned)std::min<int64_t>((work + 255) / 256, (int64_t)num_sms(device) * 8);
  if (vec) launch_pdl(true, splitk_reduce_kernel<true>, grid, 256, 0, st, ws, C, M, N, ldc, ks);
  else launch_pdl(true, splitk_reduce_kernel<false>, grid, 256, 0, st, ws, C, M, N, ldc, ks);
  return launch_status("splitk_reduce_kernel");
}

// C[b] = op(A[b]) @ op(B[b]).  a_mn_major: A stored K x M (lda = row stride of
// that storage); b_k_major: B stored N x K.
int gemm_tc(const void *A, const void *B, void *C, int c_f32, int64_t M, int64_t N, int64_t K, int64_t lda,
            int64_t ldb, int64_t ldc, int64_t batch, int64_t sA, int64_t sB, int64_t sC, int a_mn_major, int b_k_major,
            cudaStream_t st, int device, int epi = 0, int64_t n_half = 0, const void *res = nullptr, int64_t ldr = 0,
            const Args *rope = nullptr, const SymmAr *ar = nullptr, const void *ar_res = nullptr, int ksplit = 1,
            float *ws = nullptr) {
  if (M == 0 || N == 0 || batch == 0) return NKB_OK;
  if (K == 0) return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: K == 0 takes the strided path");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(NKB_ERR_UNSUPPORTED, "gemm: dims exceed int32");
  // broadcast operands (batch stride 0) reuse batch index 0 via a size-1 batch dim
  const uint64_t ba = sA ? batch : 1, bb = sB ? batch : 1;
  CUtensorMap ma, mb;
  int s;
  if (!a_mn_major) s = make_map(&ma, A, K, M, ba, lda, sA, BK, BM);
  else s = make_map(&ma, A, M, K, ba, lda, sA, 64, BK);
  if (s) return s;
  if (epi == 2 && (c_f32 || batch != 1 || !res || ldr < N))
    return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: residual epilogue needs bf16 output, one batch and a residual of N columns");
  if (epi == 1 && (b_k_major || c_f32 || n_half % 64 || N != n_half))
    return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: SwiGLU epilogue needs N-major B, bf16 output and n_half % 64 == 0");
  const int64_t bcols = epi == 1 ? 2 * n_half : N;
  // CTA pairs (256 x 256 tiles) for products with more than one row tile and no
  // split; NKB_GEMM_PAIR=0 keeps single CTAs (comparisons)
  const char *pe = getenv("NKB_GEMM_PAIR");
  const bool pair = ksplit <= 1 && M > BM && !(pe && pe[0] == '0');
  if (b_k_major) s = make_map(&mb, B, K, bcols, bb, ldb, sB, BK, pair ? BN / 2 : BN);
  else s = make_map(&mb, B, bcols, K, bb, ldb, sB, 64, BK);
  if (s) return s;
  Args args;
  args.C = C;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldc = ldc;
  args.sC = sC;
  args.batch = batch;
  args.c_f32 = c_f32;
  args.a_mn_major = a_mn_major;
  args.b_k_major = b_k_major;
  args.a_bcast = sA == 0 && batch > 1;  // one operand matrix shared by every batch (its map has one)
  args.b_bcast = sB == 0 && batch > 1;
  args.epi = epi;
  args.n_half = n_half;
  args.res = static_cast<const __nv_bfloat16 *>(res);
  args.ldr = ldr;
  args.ksplit = 1;
  args.ws = nullptr;
  if (ksplit > 1) {
    if (epi != 0 || c_f32 || batch != 1 || ar || !ws || (reinterpret_cast<uintptr_t>(ws) & 15) ||
        ksplit > (K + BK - 1) / BK)
      return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: split-K needs a plain bf16 product, one batch, a workspace and "
                                       "at most one split per k-block");
    args.ksplit = ksplit;
    args.ws = ws;
  }
  if (epi == 3) {
    if (!rope || c_f32 || batch != 1 || (rope->rope_hd != 64 && rope->rope_hd != 128) || rope->rope_seq <= 0)
      return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: rotary epilogue needs bf16 output, one batch, head_dim 64 or 128");
    if ((reinterpret_cast<uintptr_t>(rope->rope_cos) | reinterpret_cast<uintptr_t>(rope->rope_sin)) & 15)
      return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: rotary tables must be 16-byte aligned");
    for (int i = 0; i < 2; ++i)
      if (rope->rope_r0[i] % rope->rope_hd || rope->rope_r1[i] % rope->rope_hd || rope->rope_r1[i] > N)
        return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: rotary column ranges must be whole heads");
    args.rope_cos = rope->rope_cos;
    args.rope_sin = rope->rope_sin;
    for (int i = 0; i < 2; ++i) {
      args.rope_r0[i] = rope->rope_r0[i];
      args.rope_r1[i] = rope->rope_r1[i];
    }
    args.rope_hd = rope->rope_hd;
    args.rope_seq = rope->rope_seq;
  }
  args.tiles_m = (int)((M + BM - 1) / BM);
  args.tiles_m2 = (int)((M + 2 * BM - 1) / (2 * BM));
  args.tiles_n = (int)((N + (epi == 1 ? BN / 2 : BN) - 1) / (epi == 1 ? BN / 2 : BN));
  const int64_t tiles = (int64_t)args.tiles_m * args.tiles_n * batch;
  if (tiles > INT32_MAX) return fail(NKB_ERR_UNSUPPORTED, "gemm: too many tiles");
  // raster group: 2048 rows of tiles (NKB_GEMM_GROUP overrides, in row tiles)
  {
    const char *ge = getenv("NKB_GEMM_GROUP");
    const int g = ge ? atoi(ge) : 0;
    args.group = g > 0 ? g : (pair ? 8 : 16);
  }
  static ContextOnce attr_set;
  if (int s = attr_set.run(device, []() -> int {
        NKB_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tcgen05<false, false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        NKB_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tcgen05<true, false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        NKB_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tcgen05<false, true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        NKB_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_tcgen05<true, true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        return NKB_OK;
      }))
    return s;
  // one CTA per SM: every CTA of the fused kernel is resident at once, so its
  // all-reduce warps can wait for tiles of other CTAs
  const int grid = (int)std::min<int64_t>(tiles * args.ksplit, num_sms(device));
  if (ar) {
    if (epi != 0 || c_f32 || batch != 1 || ldc != N || N % 8 || args.tiles_m > SYMM_AR_CHUNKS)
      return fail(NKB_ERR_UNSUPPORTED, "gemm_tc: fused all-reduce needs a dense bf16 C, one batch, no epilogue");
    args.ar_mc = ar->mc_payload;
    args.ar_flags = ar->flags;
    args.ar_mc_flags = ar->mc_flags;
    args.ar_res = static_cast<const __nv_bfloat16 *>(ar_res);
    args.ar_rank = ar->rank;
    args.ar_world = ar->world;
    args.ar_wait = wait_limit_cycles();
    if (!pair) gemm_bf16_tcgen05<true, false><<<grid, AR_THREADS, SMEM_BYTES, st>>>(ma, mb, args);
  }
  if (pair) {
    // one cluster of two CTAs per pair of SMs, persistent over the 256 x 256 tiles
    const int64_t ptiles = (int64_t)args.tiles_m2 * args.tiles_n * batch;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(ar ? AR_THREADS : THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // as many pairs as can be resident at once (clusters stay inside a GPC); the
    // fused all-reduce relies on every CTA being resident
    static ContextOnce occ;
    static int max_clusters[64][2];
    const int dslot = device >= 0 && device < 64 ? device : 0;
    if (int s = occ.run(device, [&]() -> int {
          for (int v = 0; v < 2; ++v) {
            cudaLaunchConfig_t c = cfg;
            c.blockDim = dim3(v ? AR_THREADS : THREADS);
            c.gridDim = dim3((unsigned)num_sms(device));
            int n = 0;
            if (v)
              NKB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, gemm_bf16_tcgen05<true, true>, &c));
            else
              NKB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, gemm_bf16_tcgen05<false, true>, &c));
            max_clusters[dslot][v] = std::max(1, n);
          }
          return NKB_OK;
        }))
      return s;
    cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(ptiles, max_clusters[dslot][ar ? 1 : 0])));
    if (ar)
      NKB_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_bf16_tcgen05<true, true>, ma, mb, args));
    else
      NKB_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_bf16_tcgen05<false, true>, ma, mb, args));
  } else if (!ar) {
    gemm_bf16_tcgen05<false, false><<<grid, THREADS, SMEM_BYTES, st>>>(ma, mb, args);
  }
  if (int e = launch_status("gemm_bf16_tcgen05")) return e;
  if (args.ksplit > 1) return splitk_reduce(ws, static_cast<__nv_bfloat16 *>(C), M, N, ldc, args.ksplit, st, device);
  return NKB_OK;
}

// ---------------------------------------------------------------------------
// strided fallback: any float dtypes, arbitrary element strides, fp32
// accumulation on CUDA cores.  Used for fp32 dots (the bf16 tensor-core path
// would lose the fp32 tolerance) and for operands TMA cannot describe.
// ---------------------------------------------------------------------------
struct SimtArgs {
  const void *A, *B;
  void *C;
  int adt, bdt, cdt;
  int64_t M, N, K, batch;
  int64_t a_rs, a_cs, b_rs, b_cs, c_rs, c_cs, sA, sB, sC;
};

__global__ void __launch_bounds__(256) gemm_simt_kernel(const __grid_constant__ SimtArgs p) {
  constexpr int T = 64, TK = 16;
  __shared__ float As[TK][T + 1];
  __shared__ float Bs[TK][T + 1];
  const int64_t bz = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * T, n0 = (int64_t)blockIdx.x * T;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.K; k0 += TK) {
    for (int i = threadIdx.x; i < T * TK; i += 256) {
      const int mm = i / TK, kk = i % TK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < p.M && gk < p.K)
                       ? load_as_float(p.A, bz * p.sA + gm * p.a_rs + gk * p.a_cs, p.adt)
                       : 0.f;
      const int nn = i % T, kb = i / T;
      const int64_t gn = n0 + nn, gk2 = k0 + kb;
      Bs[kb][nn] = (gn < p.N && gk2 < p.K)
                       ? load_as_float(p.B, bz * p.sB + gk2 * p.b_rs + gn * p.b_cs, p.bdt)
                       : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < p.M && gn < p.N)
        store_from_reg(p.C, bz * p.sC + gm * p.c_rs + gn * p.c_cs, p.cdt,
                       dtype_is_float(p.cdt) ? __float_as_uint(acc[i][j]) : (uint32_t)__float2int_rn(acc[i][j]));
    }
}

int gemm_simt(const SimtArgs &p, cudaStream_t st) {
  if (p.M == 0 || p.N == 0 || p.batch == 0) return NKB_OK;
  if (p.batch > 65535) return fail(NKB_ERR_UNSUPPORTED, "gemm_simt: batch too large");
  dim3 grid((unsigned)((p.N + 63) / 64), (unsigned)((p.M + 63) / 64), (unsigned)p.batch);
  if (grid.y > 65535) return fail(NKB_ERR_UNSUPPORTED, "gemm_simt: M too large");
  gemm_simt_kernel<<<grid, 256, 0, st>>>(p);
  return launch_status("gemm_simt_kernel");
}

// ---- plan steps ---------------------------------------------------------------
// "gemm_bf16": ptrs A B C [R | COS SIN]; ints M N K lda ldb ldc batch sA sB sC c_f32 a_mn_major b_k_major
//              [epi n_half]  (epi 1: SwiGLU over [gate | up] halves of n_half columns)
//              [epi ldr]     (epi 2, fourth pointer R: C = A @ B + R, R row stride ldr)
//              [epi hd seq q0 q1 k0 k1]  (epi 3, pointers COS SIN: rotary embedding of
//                            the heads in columns [q0, q1) and [k0, k1))
//              [epi ksplit]  (epi 4, pointer WS: split-K over ksplit k-ranges, fp32
//                            partials in WS (ksplit * M * N floats), then summed)
int tc_check(const Step &s) {
  const size_t n = s.ints.size();
  if (n != 13 && n != 15 && n != 20) return fail(NKB_ERR_PLAN, "gemm_bf16: bad parameters");
  const int epi = n > 13 ? (int)s.ints[13] : 0;
  if ((epi == 3) != (n == 20)) return fail(NKB_ERR_PLAN, "gemm_bf16: bad epilogue parameters");
  const size_t ptrs = (epi == 2 || epi == 4) ? 4u : epi == 3 ? 5u : 3u;
  if (s.buf_ids.size() != ptrs) return fail(NKB_ERR_PLAN, "gemm_bf16: bad pointer count");
  if (epi < 0 || epi > 4) return fail(NKB_ERR_PLAN, "gemm_bf16: unknown epilogue");
  if (epi == 4 && s.ints[14] < 2) return fail(NKB_ERR_PLAN, "gemm_bf16: split-K needs two or more splits");
  return NKB_OK;
}
int tc_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  const int epi = q.size() > 13 ? (int)q[13] : 0;
  const int64_t n_half = epi == 1 ? q[14] : 0;
  const int64_t ldr = epi == 2 ? q[14] : 0;
  Args rope;
  if (epi == 3) {
    rope.rope_cos = static_cast<const __nv_bfloat16 *>(a.ptrs[3]);
    rope.rope_sin = static_cast<const __nv_bfloat16 *>(a.ptrs[4]);
    rope.rope_hd = (int)q[14];
    rope.rope_seq = (int)q[15];
    rope.rope_r0[0] = q[16];
    rope.rope_r1[0] = q[17];
    rope.rope_r0[1] = q[18];
    rope.rope_r1[1] = q[19];
  }
  if (epi == 4)
    return gemm_tc(a.ptrs[0], a.ptrs[1], a.ptrs[2], (int)q[10], q[0], q[1], q[2], q[3], q[4], q[5], q[6], q[7], q[8],
                   q[9], (int)q[11], (int)q[12], a.stream, a.device, 0, 0, nullptr, 0, nullptr, nullptr, nullptr,
                   (int)q[14], static_cast<float *>(a.ptrs[3]));
  return gemm_tc(a.ptrs[0], a.ptrs[1], a.ptrs[2], (int)q[10], q[0], q[1], q[2], q[3], q[4], q[5], q[6], q[7], q[8],
                 q[9], (int)q[11], (int)q[12], a.stream, a.device, epi, n_half, epi == 2 ? a.ptrs[3] : nullptr, ldr,
                 epi == 3 ? &rope : nullptr);
}

// "gemm_bf16_ar": ptrs A B C [R]; ints M N K lda ldb ldc batch sA sB sC c_f32 a_mn_major b_k_major slot.
// C (bf16, dense) lies in the plan's symmetric region; afterwards it holds the
// sum over the ranks of A @ B (+ R when given, R dense with N columns).  With a
// bound symmetric region the reduction runs inside the GEMM kernel (flag slot
// `slot`); otherwise the GEMM is followed by the communicator's all-reduce.
int ar_check(const Step &s) {
  if (s.ints.size() != 14 || (s.buf_ids.size() != 3 && s.buf_ids.size() != 4))
    return fail(NKB_ERR_PLAN, "gemm_bf16_ar: bad parameters");
  if (s.ints[13] < 0 || s.ints[13] >= SYMM_AR_SLOTS) return fail(NKB_ERR_PLAN, "gemm_bf16_ar: bad flag slot");
  if (s.ints[10] != 0 || s.ints[6] != 1 || s.ints[5] != s.ints[1])
    return fail(NKB_ERR_PLAN, "gemm_bf16_ar: C must be dense bf16, one batch");
  return NKB_OK;
}
int ar_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  const void *res = a.step->buf_ids.size() == 4 ? a.ptrs[3] : nullptr;
  const int64_t M = q[0], N = q[1];
  const size_t count = (size_t)M * N;
  SymmAr ar;
  const bool fused = a.comm && M > 0 && N % 8 == 0 && (M + BM - 1) / BM <= SYMM_AR_CHUNKS &&
                     ((reinterpret_cast<uintptr_t>(res) & 15) == 0) &&
                     comm_symm_ar(a.comm, a.ptrs[2], count * 2, (int)q[13], &ar);
  if (int s = gemm_tc(a.ptrs[0], a.ptrs[1], a.ptrs[2], 0, M, N, q[2], q[3], q[4], q[5], 1, q[7], q[8], q[9],
                      (int)q[11], (int)q[12], a.stream, a.device, 0, 0, nullptr, 0, nullptr, fused ? &ar : nullptr,
                      res))
    return s;
  if (fused) return NKB_OK;
  if (!a.comm) return fail(NKB_ERR_STATE, "gemm_bf16_ar: no communicator is bound to the plan");
  if (res) return comm_all_reduce_add(a.comm, a.ptrs[2], res, a.ptrs[2], count, NKB_BF16, a.stream);
  return comm_all_reduce(a.comm, a.ptrs[2], a.ptrs[2], count, NKB_BF16, a.stream);
}

// "gemm_simt": ptrs A B C; ints adt bdt cdt M N K batch a_rs a_cs b_rs b_cs c_rs c_cs sA sB sC
int simt_check(const Step &s) {
  if (s.buf_ids.size() != 3 || s.ints.size() != 16) return fail(NKB_ERR_PLAN, "gemm_simt: bad parameters");
  return NKB_OK;
}
int simt_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  SimtArgs p;
  p.A = a.ptrs[0];
  p.B = a.ptrs[1];
  p.C = a.ptrs[2];
  p.adt = (int)q[0];
  p.bdt = (int)q[1];
  p.cdt = (int)q[2];
  p.M = q[3];
  p.N = q[4];
  p.K = q[5];
  p.batch = q[6];
  p.a_rs = q[7];
  p.a_cs = q[8];
  p.b_rs = q[9];
  p.b_cs = q[10];
  p.c_rs = q[11];
  p.c_cs = q[12];
  p.sA = q[13];
  p.sB = q[14];
  p.sC = q[15];
  return gemm_simt(p, a.stream);
}

}  // namespace gemm

NKB_REGISTER_KERNEL("gemm_bf16", gemm::tc_launch, gemm::tc_check);
NKB_REGISTER_KERNEL("gemm_simt", gemm::simt_launch, gemm::simt_check);
NKB_REGISTER_KERNEL("gemm_bf16_ar", gemm::ar_launch, gemm::ar_check);

// Device error flag of the bounded waits (read by nkb_check_device_error).
int gemm_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, gemm::g_device_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(gemm::g_device_error, &zero, sizeof(int)));
  return NKB_OK;
}

}  // namespace nkb

extern "C" int nkb_gemm_bf16(const void *A, const void *B, void *C, int c_dtype, int64_t M, int64_t N, int64_t K,
                             int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t sA, int64_t sB, int64_t sC,
                             void *stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c_dtype != NKB_BF16 && c_dtype != NKB_F32) return nkb::fail(NKB_ERR_UNSUPPORTED, "gemm: output must be bf16 or fp32");
  if (K > 0 && nkb::gemm::tc_eligible(A, B, lda, ldb, sA, sB, batch) && (batch == 1 || (sA && sB)))
    return nkb::gemm::gemm_tc(A, B, C, c_dtype == NKB_F32, M, N, K, lda, ldb, ldc, batch, sA, sB, sC, 0, 0, st, dev);
  nkb::gemm::SimtArgs p{A, B, C, NKB_BF16, NKB_BF16, c_dtype, M, N, K, batch, lda, 1, ldb, 1, ldc, 1, sA, sB, sC};
  return nkb::gemm::gemm_simt(p, st);
}
