// Layout moves whose innermost axis changes (a materialised np.transpose,
// core/ops/transform.py:55-79, and any permuted copy the planner folds into
// one), staged through shared memory by TMA.
//
// The move is a batched 2-D transpose: the input's contiguous axis C and the
// output's contiguous axis R trade places, up to three further axes are a
// batch with their own input and output strides.  Square tiles of
// T = 128 / esize elements (128 bytes a row) are loaded by
// cp.async.bulk.tensor with the 128-byte swizzle, transposed in registers by
// blocks of V x V elements (V = 16 / esize: one 16-byte vector a row), written
// into an output tile in the same swizzled layout and stored by
// cp.async.bulk.tensor.  Ragged edges need no code: the load fills zeros
// outside the input and the store clips at the output's bounds.
//
// Shared-memory banks: a warp's 16-byte accesses run in phases of 8 threads.
// Thread (phase p, slot k) takes the block of row group rb = k and chunk
// c = k ^ p; in the swizzled layout its loads hit chunk c ^ ((V rb + q) & 7)
// and its stores chunk rb ^ ((V c + e) & 7), which are 8 different chunks in
// every phase for esize 2 and 4 (and 1 and 8), so neither side has bank
// conflicts.  Traced kernels carry no 8-byte types (64-bit inputs are
// down-cast at trace time) and 1-byte moves keep the elementwise copy, so the
// kernel is built for 2- and 4-byte elements.
//
// A persistent grid of 256-thread CTAs, each four independent teams of 64
// threads; team k of CTA b takes tiles 4b + k, 4b + k + 4 * grid, ...
// (consecutive tiles along R, so the four teams of a CTA fill 512 contiguous
// bytes of each output row), with 4 load stages in flight and two output
// buffers of its own, its first thread issuing its copies, and only its own
// named barrier between them.  All waits are bounded; on expiry the team
// raises the device error flag, lets copies still in flight land, and
// returns.  No cluster multicast anywhere.
#include "sm100.cuh"

namespace nkb {
namespace tr {

using namespace sm100;

constexpr int THREADS = 256, TILES = 4, STAGES = 4, OUTBUF = 2;
__device__ int g_error = 0;

struct Params {
  int64_t n_tiles;
  int n_c, n_r;  // tiles along C (the input's contiguous axis) and R (the output's)
  int bdim[3];   // batch extents (1 when absent)
};

template <int E>
struct Geo {
  static constexpr int V = 16 / E;          // elements per 16-byte vector
  static constexpr int T = 128 / E;         // tile edge in elements
  static constexpr int TILE_BYTES = T * 128;
};

template <int RANK>
__device__ __forceinline__ void tma_load(void *dst, const CUtensorMap *m, uint64_t *bar, const int *c) {
  if constexpr (RANK == 2)
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c[0]), "r"(c[1])
        : "memory");
  else if constexpr (RANK == 3)
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c[0]), "r"(c[1]),
        "r"(c[2])
        : "memory");
  else if constexpr (RANK == 4)
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c[0]), "r"(c[1]),
        "r"(c[2]), "r"(c[3])
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
        "%7}], [%2];" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c[0]),
        "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4])
        : "memory");
}

template <int RANK>
__device__ __forceinline__ void tma_store(const CUtensorMap *m, const void *src, const int *c) {
  if constexpr (RANK == 2)
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)), "r"(smem_u32(src)), "r"(c[0]), "r"(c[1])
                 : "memory");
  else if constexpr (RANK == 3)
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)), "r"(smem_u32(src)), "r"(c[0]), "r"(c[1]), "r"(c[2])
                 : "memory");
  else if constexpr (RANK == 4)
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)), "r"(smem_u32(src)), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3])
                 : "memory");
  else
    asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)), "r"(smem_u32(src)), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]),
                 "r"(c[4])
                 : "memory");
}

// Coordinates of tile t: x along the contiguous axis of the map, y along the
// other transposed axis, then the batch coordinates.
__device__ __forceinline__ void tile_coords(const Params &p, int64_t t, int T, int *in_c, int *out_c) {
  const int rt = (int)(t % p.n_r);
  int64_t u = t / p.n_r;
  const int ct = (int)(u % p.n_c);
  u /= p.n_c;
  const int z0 = (int)(u % p.bdim[0]);
  u /= p.bdim[0];
  const int z1 = (int)(u % p.bdim[1]);
  const int z2 = (int)(u / p.bdim[1]);
  in_c[0] = ct * T, in_c[1] = rt * T, in_c[2] = z0, in_c[3] = z1, in_c[4] = z2;
  out_c[0] = rt * T, out_c[1] = ct * T, out_c[2] = z0, out_c[3] = z1, out_c[4] = z2;
}

// V x V block transpose of V row vectors (16 bytes each) into V column vectors.
template <int E>
__device__ __forceinline__ void block_transpose(const uint4 *v, uint4 *w) {
  if constexpr (E == 4) {
    const uint32_t *a = reinterpret_cast<const uint32_t *>(v);
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = make_uint4(a[e], a[4 + e], a[8 + e], a[12 + e]);
  } else {  // E == 2: element e of row q is half (e & 1) of word e >> 1
    const uint32_t *a = reinterpret_cast<const uint32_t *>(v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = __byte_perm(a[(2 * k) * 4 + (e >> 1)], a[(2 * k + 1) * 4 + (e >> 1)], sel);
      w[e] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// bar.sync over `threads` threads on barrier `id`, returning the AND of `pred`
__device__ __forceinline__ bool team_and(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void team_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Four independent teams of 64 threads per CTA, each a pipeline of its own:
// STAGES input tiles and OUTBUF output tiles, its leader (first thread)
// issuing its copies; a team synchronises on its own named barrier only.
template <int E, int RANK>
__global__ void __launch_bounds__(THREADS) transpose_tiles_kernel(const __grid_constant__ CUtensorMap min,
                                                                  const __grid_constant__ CUtensorMap mout,
                                                                  const __grid_constant__ Params p) {
  using G = Geo<E>;
  constexpr int TEAM = THREADS / TILES;  // 64 threads: one 16-byte block of the tile each
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[TILES][STAGES];
  __shared__ int abort_flag[TILES];

  const int tid = threadIdx.x, team = tid / TEAM, unit = tid % TEAM;
  const bool leader = unit == 0;
  uint8_t *in_buf = smem + team * (STAGES + OUTBUF) * G::TILE_BYTES;  // [STAGES][TILE_BYTES]
  uint8_t *out_buf = in_buf + STAGES * G::TILE_BYTES;                 // [OUTBUF][TILE_BYTES]
  const int64_t first = (int64_t)blockIdx.x * TILES + team, step = (int64_t)gridDim.x * TILES;
  if (leader) {
    if (team == 0) {
      prefetch_map(&min);
      prefetch_map(&mout);
    }
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[team][s], 1);
    abort_flag[team] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  auto issue_load = [&](int64_t t, int s) {
    int ic[5], oc[5];
    tile_coords(p, t, G::T, ic, oc);
    mbar_expect_tx(&full[team][s], (uint32_t)G::TILE_BYTES);
    tma_load<RANK>(in_buf + s * G::TILE_BYTES, &min, &full[team][s], ic);
  };
  if (leader)
    for (int s = 0; s < STAGES; ++s)
      if (first + s * step < p.n_tiles) issue_load(first + s * step, s);

  // this thread's V x V block of the tile
  const int rb = unit & 7, c = (unit & 7) ^ (unit >> 3);
  int it = 0;
  for (int64_t t = first; t < p.n_tiles; t += step, ++it) {
    const int s = it % STAGES, ob = it % OUTBUF;
    bool ok = mbar_wait(&full[team][s], (it / STAGES) & 1, &abort_flag[team], &g_error);
    if (leader) bulk_wait_read<OUTBUF - 1>();  // the store that last read out_buf[ob] is done with it
    // one decision for the whole team, so that its threads meet the same barriers
    if (!team_and(1 + team, TEAM, ok)) break;
    const uint8_t *src = in_buf + s * G::TILE_BYTES;
    uint8_t *dst = out_buf + ob * G::TILE_BYTES;
    uint4 v[G::V], w[G::V];
#pragma unroll
    for (int q = 0; q < G::V; ++q) {
      const int row = G::V * rb + q;
      v[q] = *reinterpret_cast<const uint4 *>(src + row * 128 + ((c ^ (row & 7)) << 4));
    }
    block_transpose<E>(v, w);
#pragma unroll
    for (int e = 0; e < G::V; ++e) {
      const int row = G::V * c + e;
      *reinterpret_cast<uint4 *>(dst + row * 128 + ((rb ^ (row & 7)) << 4)) = w[e];
    }
    fence_proxy_async_smem();
    team_sync(1 + team, TEAM);
    if (leader) {
      int ic[5], oc[5];
      tile_coords(p, t, G::T, ic, oc);
      tma_store<RANK>(&mout, dst, oc);
      bulk_commit();
      const int64_t next = t + STAGES * step;  // every thread of the team has read stage s: refill it
      if (next < p.n_tiles) issue_load(next, s);
    }
  }
  if (leader) {
    bulk_wait<0>();
    if (abort_flag[team]) {
      // bounded drain of loads that may still be landing in shared memory
      const long long t0 = clock64();
      while (clock64() - t0 < 2000000) {
      }
    }
  }
  __syncthreads();
}

// Step layout ("transpose_tiles"): ptrs src dst; ints
//   esize C R src_stride_R dst_stride_C nb [extent src_stride dst_stride] x nb
// (elements).  C is the source's contiguous axis (stride 1), R the
// destination's; C has stride dst_stride_C in the destination and R stride
// src_stride_R in the source.
int check(const Step &s) {
  const auto &q = s.ints;
  if (s.buf_ids.size() != 2 || q.size() < 6) return fail(NKB_ERR_PLAN, "transpose_tiles: bad parameters");
  const int64_t E = q[0], nb = q[5];
  if (E != 2 && E != 4) return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: element size 2 or 4");
  if (nb < 0 || nb > 3 || (int64_t)q.size() != 6 + 3 * nb) return fail(NKB_ERR_PLAN, "transpose_tiles: batch axes");
  if (q[1] <= 0 || q[2] <= 0 || q[1] >= (1LL << 31) || q[2] >= (1LL << 31))
    return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: extents");
  if ((q[3] * E) % 16 || (q[4] * E) % 16 || q[3] <= 0 || q[4] <= 0)
    return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: strides must be positive multiples of 16 bytes");
  for (int i = 0; i < nb; ++i) {
    const int64_t ext = q[6 + 3 * i], ss = q[7 + 3 * i], ds = q[8 + 3 * i];
    if (ext <= 0 || ext >= (1LL << 31) || ss <= 0 || ds <= 0 || (ss * E) % 16 || (ds * E) % 16)
      return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: batch extents/strides");
  }
  return NKB_OK;
}

CUtensorMapDataType map_type(int E) {
  return E == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
}

int make_map(CUtensorMap *m, const void *base, int E, int rank, const uint64_t *dims, const uint64_t *strides_bytes) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(NKB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: base not 16-byte aligned");
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t box[5], es[5];
  const uint32_t T = 128 / E;
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    box[i] = i < 2 ? T : 1;
    es[i] = 1;
    if (i > 0) gstride[i - 1] = strides_bytes[i - 1];
  }
  CUresult r = enc(m, map_type(E), rank, const_cast<void *>(base), gdim, gstride, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NKB_ERR_UNSUPPORTED, "transpose_tiles: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return NKB_OK;
}

template <int E, int RANK>
int run(const CUtensorMap &mi, const CUtensorMap &mo, const Params &p, int device, cudaStream_t stream) {
  constexpr int SMEM = (STAGES + OUTBUF) * TILES * Geo<E>::TILE_BYTES + 1024;  // four teams
  static ContextOnce attr;
  if (int s = attr.run(device, []() -> int {
        NKB_CUDA_TRY(
            cudaFuncSetAttribute(transpose_tiles_kernel<E, RANK>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        return NKB_OK;
      }))
    return s;
  const int per_sm = (227 * 1024) / SMEM;
  const int64_t grid =
      std::min<int64_t>((p.n_tiles + TILES - 1) / TILES, (int64_t)num_sms(device) * std::max(1, per_sm));
  transpose_tiles_kernel<E, RANK><<<(unsigned)grid, THREADS, SMEM, stream>>>(mi, mo, p);
  return launch_status("transpose_tiles_kernel");
}

template <int E>
int run_rank(int rank, const CUtensorMap &mi, const CUtensorMap &mo, const Params &p, int device, cudaStream_t st) {
  switch (rank) {
    case 2: return run<E, 2>(mi, mo, p, device, st);
    case 3: return run<E, 3>(mi, mo, p, device, st);
    case 4: return run<E, 4>(mi, mo, p, device, st);
    default: return run<E, 5>(mi, mo, p, device, st);
  }
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  const int E = (int)q[0], nb = (int)q[5], rank = 2 + nb;
  const int64_t C = q[1], R = q[2];
  uint64_t din[5] = {(uint64_t)C, (uint64_t)R}, dout[5] = {(uint64_t)R, (uint64_t)C};
  uint64_t sin[4] = {(uint64_t)(q[3] * E)}, sout[4] = {(uint64_t)(q[4] * E)};
  Params p{};
  p.bdim[0] = p.bdim[1] = p.bdim[2] = 1;
  int64_t nbatch = 1;
  for (int i = 0; i < nb; ++i) {
    din[2 + i] = dout[2 + i] = (uint64_t)q[6 + 3 * i];
    sin[1 + i] = (uint64_t)(q[7 + 3 * i] * E);
    sout[1 + i] = (uint64_t)(q[8 + 3 * i] * E);
    p.bdim[i] = (int)q[6 + 3 * i];
    nbatch *= q[6 + 3 * i];
  }
  const int T = 128 / E;
  p.n_c = (int)((C + T - 1) / T);
  p.n_r = (int)((R + T - 1) / T);
  const int64_t n_tiles = (int64_t)p.n_c * p.n_r * nbatch;
  if (!n_tiles) return NKB_OK;
  p.n_tiles = n_tiles;
  CUtensorMap mi, mo;
  if (int s = make_map(&mi, a.ptrs[0], E, rank, din, sin)) return s;
  if (int s = make_map(&mo, a.ptrs[1], E, rank, dout, sout)) return s;
  return E == 2 ? run_rank<2>(rank, mi, mo, p, a.device, a.stream) : run_rank<4>(rank, mi, mo, p, a.device, a.stream);
}

}  // namespace tr

int transpose_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, tr::g_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(tr::g_error, &zero, sizeof(int)));
  return NKB_OK;
}

NKB_REGISTER_KERNEL("transpose_tiles", tr::launch, tr::check);

}  // namespace nkb
