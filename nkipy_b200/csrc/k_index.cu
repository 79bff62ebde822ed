// Index kernels (bit-exact data movement) and the collective step.
//
//  take        HLO gather with one collapsed axis, as np.take / tensor
//              indexing traces it (reference core/ops/indexing.py:115-205):
//              out[p, j, q] = x[p, clamp(idx[j]), q];
//  gather_pts  point gather with full index vectors, as take_along_axis
//              traces it (indexing.py:214-353): out[i] = x[clamp(idx[i, :])];
//  pad         HLO pad with a constant value (transform.py:506-560);
//  scatter     HLO scatter with update_computation "assign" of whole windows
//              along one axis (indexing.py:360-433) or of points
//              (indexing.py:771-862);
//  allreduce   HLO all-reduce (collectives.py:87-110), sum: inside NVSwitch when the
//              payload sits in the communicator's symmetric region, else NCCL;
//  allreduce_add  the same followed by the residual add of a row-parallel block.
// Indices are clamped into range like XLA gather/scatter start indices, so no
// index value can address memory outside the operand.

#include "common.cuh"

namespace nkb {
namespace idx {

__device__ __forceinline__ int64_t clamp_index(int64_t v, int64_t n) { return v < 0 ? 0 : (v >= n ? n - 1 : v); }

__device__ __forceinline__ int64_t load_index(const void *p, int64_t i, int dt) {
  const uint32_t raw = load_as_reg(p, i, dt);
  return (dt == NKB_U32 || dt == NKB_U16 || dt == NKB_U8) ? (int64_t)raw : (int64_t)(int32_t)raw;
}

__global__ void take_kernel(const uint8_t *__restrict__ x, const void *__restrict__ ind, int ind_dt,
                            uint8_t *__restrict__ out, int64_t pre, int64_t axis_len, int64_t post_bytes, int64_t n_idx) {
  // one CTA row per (p, j); threads copy the contiguous post block bytewise in 16B/1B pieces
  for (int64_t r = blockIdx.x; r < pre * n_idx; r += gridDim.x) {
    const int64_t p = r / n_idx, j = r - p * n_idx;
    const int64_t src_row = clamp_index(load_index(ind, j, ind_dt), axis_len);
    const uint8_t *src = x + (p * axis_len + src_row) * post_bytes;
    uint8_t *dst = out + r * post_bytes;
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | post_bytes) & 15) == 0) {
      for (int64_t b = threadIdx.x * 16; b < post_bytes; b += blockDim.x * 16)
        *reinterpret_cast<uint4 *>(dst + b) = *reinterpret_cast<const uint4 *>(src + b);
    } else {
      for (int64_t b = threadIdx.x; b < post_bytes; b += blockDim.x) dst[b] = src[b];
    }
  }
}

constexpr int kMaxRank = 8;
struct PtsParams {
  const uint8_t *x;
  const void *ind;
  uint8_t *out;
  int ind_dt, rank, esize;
  int64_t n;
  int64_t shape[kMaxRank], strides[kMaxRank];
};

__global__ void gather_pts_kernel(const __grid_constant__ PtsParams p) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t off = 0;
    for (int d = 0; d < p.rank; ++d) off += clamp_index(load_index(p.ind, i * p.rank + d, p.ind_dt), p.shape[d]) * p.strides[d];
    const uint8_t *src = p.x + off * p.esize;
    uint8_t *dst = p.out + i * p.esize;
    for (int b = 0; b < p.esize; ++b) dst[b] = src[b];
  }
}

struct PadParams {
  const uint8_t *x;
  uint8_t *out;
  int rank, esize;
  int64_t n;
  int64_t in_shape[kMaxRank], out_shape[kMaxRank], lo[kMaxRank];
  uint32_t value_bits;
};

__global__ void pad_kernel(const __grid_constant__ PadParams p) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, src = 0, mul = 1;
    bool inside = true;
    for (int d = p.rank - 1; d >= 0; --d) {
      const int64_t od = rem % p.out_shape[d];
      rem /= p.out_shape[d];
      const int64_t id = od - p.lo[d];
      if (id < 0 || id >= p.in_shape[d]) inside = false;
      src += id * mul;
      mul *= p.in_shape[d];
    }
    uint8_t *dst = p.out + i * p.esize;
    if (inside) {
      for (int b = 0; b < p.esize; ++b) dst[b] = p.x[src * p.esize + b];
    } else {
      for (int b = 0; b < p.esize; ++b) dst[b] = (uint8_t)(p.value_bits >> (8 * b));
    }
  }
}

// Window scatter along `axis` of a (pre, axis_len, post) operand; updates are
// (pre, n_idx, post), dense within each of the `pre` blocks, blocks
// `upd_pre_bytes` apart.  Duplicate indices: the last writer wins in an
// unspecified order, as for XLA with unique_indices = false.
// One launch may carry two scatters (the decode step's K and V cache rows):
// blocks [0, seg[0].blocks) take the first, the rest the second.
struct ScatterSeg {
  uint8_t *out;
  const void *ind;
  const uint8_t *upd;
  int64_t pre, axis_len, post_bytes, n_idx, upd_pre_bytes;
  int ind_dt;
  unsigned blocks;
};
struct ScatterLaunch {
  ScatterSeg seg[2];
  int nseg;
};

__global__ void scatter_rows_kernel(const __grid_constant__ ScatterLaunch L) {
  pdl_wait();
  pdl_trigger();
  const int si = (L.nseg > 1 && blockIdx.x >= L.seg[0].blocks) ? 1 : 0;
  const ScatterSeg &S = L.seg[si];
  uint8_t *__restrict__ out = S.out;
  const void *__restrict__ ind = S.ind;
  const uint8_t *__restrict__ upd = S.upd;
  const int ind_dt = S.ind_dt;
  const int64_t pre = S.pre, axis_len = S.axis_len, post_bytes = S.post_bytes, n_idx = S.n_idx,
                upd_pre_bytes = S.upd_pre_bytes;
  const int64_t bx = (int64_t)blockIdx.x - (si ? L.seg[0].blocks : 0);
  // 16-byte copies when every row start is 16-byte aligned (a KV-cache row of
  // 2 KB is one vector per thread), else bytes
  const bool vec = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(upd) | (uintptr_t)post_bytes |
                     (uintptr_t)upd_pre_bytes) & 15) == 0;
  for (int64_t r = bx; r < pre * n_idx; r += S.blocks) {
    const int64_t p = r / n_idx, j = r - p * n_idx;
    const int64_t dst_row = load_index(ind, j, ind_dt);
    if (dst_row < 0 || dst_row >= axis_len) continue;  // out-of-range updates are skipped
    uint8_t *dst = out + (p * axis_len + dst_row) * post_bytes;
    const uint8_t *src = upd + p * upd_pre_bytes + j * post_bytes;
    if (vec) {
      const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll 4
      for (int64_t b = threadIdx.x; b < post_bytes / 16; b += blockDim.x) d4[b] = s4[b];
    } else {
      for (int64_t b = threadIdx.x; b < post_bytes; b += blockDim.x) dst[b] = src[b];
    }
  }
}

__global__ void scatter_pts_kernel(uint8_t *__restrict__ out, const void *__restrict__ ind, int ind_dt,
                                   const uint8_t *__restrict__ upd, int rank, int esize, int64_t n,
                                   PtsParams geo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t off = 0;
    bool ok = true;
    for (int d = 0; d < rank; ++d) {
      const int64_t v = load_index(ind, i * rank + d, ind_dt);
      if (v < 0 || v >= geo.shape[d]) ok = false;
      off += v * geo.strides[d];
    }
    if (!ok) continue;
    for (int b = 0; b < esize; ++b) out[off * esize + b] = upd[i * esize + b];
  }
}

unsigned grid_for(int64_t work, int device, int per_sm = 16) {
  const int64_t cap = (int64_t)num_sms(device) * per_sm;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(work, cap));
}

// "take": ptrs x idx out; ints ind_dtype pre axis_len post_bytes n_idx
int take_check(const Step &s) {
  if (s.buf_ids.size() != 3 || s.ints.size() != 5) return fail(NKB_ERR_PLAN, "take: bad parameters");
  if (s.ints[2] <= 0) return fail(NKB_ERR_UNSUPPORTED, "take: empty gather axis");
  return NKB_OK;
}
int take_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  if (q[1] * q[4] == 0 || q[3] == 0) return NKB_OK;
  take_kernel<<<grid_for(q[1] * q[4], a.device, 32), 128, 0, a.stream>>>(
      (const uint8_t *)a.ptrs[0], a.ptrs[1], (int)q[0], (uint8_t *)a.ptrs[2], q[1], q[2], q[3], q[4]);
  return launch_status("take_kernel");
}

// "gather_pts": ptrs x idx out; ints ind_dtype rank esize n shape[rank] strides[rank]
int pts_check(const Step &s) {
  if (s.buf_ids.size() != 3 || s.ints.size() < 4) return fail(NKB_ERR_PLAN, "gather_pts: bad parameters");
  const int64_t r = s.ints[1];
  if (r < 1 || r > kMaxRank || (int64_t)s.ints.size() != 4 + 2 * r) return fail(NKB_ERR_PLAN, "gather_pts: rank");
  for (int d = 0; d < r; ++d)
    if (s.ints[4 + d] <= 0) return fail(NKB_ERR_UNSUPPORTED, "gather_pts: empty operand axis");
  return NKB_OK;
}
int pts_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  PtsParams p;
  memset(&p, 0, sizeof(p));
  p.x = (const uint8_t *)a.ptrs[0];
  p.ind = a.ptrs[1];
  p.out = (uint8_t *)a.ptrs[2];
  p.ind_dt = (int)q[0];
  p.rank = (int)q[1];
  p.esize = (int)q[2];
  p.n = q[3];
  for (int d = 0; d < p.rank; ++d) {
    p.shape[d] = q[4 + d];
    p.strides[d] = q[4 + p.rank + d];
  }
  if (!p.n) return NKB_OK;
  gather_pts_kernel<<<grid_for((p.n + 255) / 256, a.device), 256, 0, a.stream>>>(p);
  return launch_status("gather_pts_kernel");
}

// "pad": ptrs x out; ints rank esize n value_bits in_shape[rank] out_shape[rank] lo[rank]
int pad_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() < 4) return fail(NKB_ERR_PLAN, "pad: bad parameters");
  const int64_t r = s.ints[0];
  if (r < 1 || r > kMaxRank || (int64_t)s.ints.size() != 4 + 3 * r) return fail(NKB_ERR_PLAN, "pad: rank");
  return NKB_OK;
}
int pad_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  PadParams p;
  memset(&p, 0, sizeof(p));
  p.x = (const uint8_t *)a.ptrs[0];
  p.out = (uint8_t *)a.ptrs[1];
  p.rank = (int)q[0];
  p.esize = (int)q[1];
  p.n = q[2];
  p.value_bits = (uint32_t)q[3];
  for (int d = 0; d < p.rank; ++d) {
    p.in_shape[d] = q[4 + d];
    p.out_shape[d] = q[4 + p.rank + d];
    p.lo[d] = q[4 + 2 * p.rank + d];
  }
  if (!p.n) return NKB_OK;
  pad_kernel<<<grid_for((p.n + 255) / 256, a.device), 256, 0, a.stream>>>(p);
  return launch_status("pad_kernel");
}

// "scatter_rows": ptrs out idx upd; ints ind_dtype pre axis_len post_bytes n_idx
// [upd_pre_bytes] (absent: the updates are dense).  Two scatters merged by the
// planner: 6 ptrs, 12 ints (both with upd_pre_bytes).
int srows_check(const Step &s) {
  const bool two = s.buf_ids.size() == 6 && s.ints.size() == 12;
  if (!two && (s.buf_ids.size() != 3 || (s.ints.size() != 5 && s.ints.size() != 6)))
    return fail(NKB_ERR_PLAN, "scatter_rows: bad parameters");
  for (size_t o = 0; o < s.ints.size(); o += 6)
    if (s.ints.size() >= o + 6 && s.ints[o + 5] < s.ints[o + 4] * s.ints[o + 3])
      return fail(NKB_ERR_PLAN, "scatter_rows: update blocks overlap");
  return NKB_OK;
}
int srows_launch(const LaunchArgs &a) {
  const auto &all = a.step->ints;
  ScatterLaunch L;
  L.nseg = all.size() == 12 ? 2 : 1;
  unsigned grid = 0;
  for (int i = 0; i < L.nseg; ++i) {
    const int64_t *q = all.data() + 6 * i;
    ScatterSeg &S = L.seg[i];
    S.out = static_cast<uint8_t *>(a.ptrs[3 * i]);
    S.ind = a.ptrs[3 * i + 1];
    S.upd = static_cast<const uint8_t *>(a.ptrs[3 * i + 2]);
    S.ind_dt = (int)q[0];
    S.pre = q[1];
    S.axis_len = q[2];
    S.post_bytes = q[3];
    S.n_idx = q[4];
    S.upd_pre_bytes = (L.nseg == 2 || all.size() == 6) ? q[5] : q[4] * q[3];
    S.blocks = (S.pre * S.n_idx == 0 || S.post_bytes == 0) ? 0u : grid_for(S.pre * S.n_idx, a.device, 32);
    grid += S.blocks;
  }
  if (grid == 0) return NKB_OK;
  launch_pdl(a.pdl, scatter_rows_kernel, grid, 128, 0, a.stream, L);
  return launch_status("scatter_rows_kernel");
}

// "scatter_pts": ptrs out idx upd; ints ind_dtype rank esize n shape[rank] strides[rank]
int spts_check(const Step &s) { return pts_check(s); }
int spts_launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  PtsParams geo;
  memset(&geo, 0, sizeof(geo));
  const int rank = (int)q[1];
  for (int d = 0; d < rank; ++d) {
    geo.shape[d] = q[4 + d];
    geo.strides[d] = q[4 + rank + d];
  }
  if (!q[3]) return NKB_OK;
  scatter_pts_kernel<<<grid_for((q[3] + 255) / 256, a.device), 256, 0, a.stream>>>(
      (uint8_t *)a.ptrs[0], a.ptrs[1], (int)q[0], (const uint8_t *)a.ptrs[2], rank, (int)q[2], q[3], geo);
  return launch_status("scatter_pts_kernel");
}

// "copy_bytes": ptrs src dst; ints bytes  (dense copy; no-op when src == dst)
int copy_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() != 1) return fail(NKB_ERR_PLAN, "copy_bytes: bad parameters");
  return NKB_OK;
}
int copy_launch(const LaunchArgs &a) {
  if (a.ptrs[0] == a.ptrs[1] || a.step->ints[0] == 0) return NKB_OK;
  NKB_CUDA_TRY(cudaMemcpyAsync(a.ptrs[1], a.ptrs[0], (size_t)a.step->ints[0], cudaMemcpyDeviceToDevice, a.stream));
  return NKB_OK;
}

// "allreduce": ptrs src dst; ints count dtype
int ar_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() != 2) return fail(NKB_ERR_PLAN, "allreduce: bad parameters");
  return NKB_OK;
}
int ar_launch(const LaunchArgs &a) {
  return comm_all_reduce(a.comm, a.ptrs[0], a.ptrs[1], (size_t)a.step->ints[0], (int)a.step->ints[1], a.stream);
}

// "allreduce_add": ptrs buf res dst; ints count dtype -- dst = res + all-reduce(buf), buf keeps the sum
int ara_check(const Step &s) {
  if (s.buf_ids.size() != 3 || s.ints.size() != 2) return fail(NKB_ERR_PLAN, "allreduce_add: bad parameters");
  if (s.ints[1] != NKB_BF16 && s.ints[1] != NKB_F32) return fail(NKB_ERR_UNSUPPORTED, "allreduce_add: bf16 or fp32");
  return NKB_OK;
}
int ara_launch(const LaunchArgs &a) {
  return comm_all_reduce_add(a.comm, a.ptrs[0], a.ptrs[1], a.ptrs[2], (size_t)a.step->ints[0], (int)a.step->ints[1],
                             a.stream);
}

// "allgather" / "reducescatter" / "alltoall": ptrs send recv; ints count (per rank / block) dtype
int coll_check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() != 2) return fail(NKB_ERR_PLAN, "allgather/reducescatter: bad parameters");
  return NKB_OK;
}
int ag_launch(const LaunchArgs &a) {
  return comm_all_gather(a.comm, a.ptrs[0], a.ptrs[1], (size_t)a.step->ints[0], (int)a.step->ints[1], a.stream);
}
int rs_launch(const LaunchArgs &a) {
  return comm_reduce_scatter(a.comm, a.ptrs[0], a.ptrs[1], (size_t)a.step->ints[0], (int)a.step->ints[1], a.stream);
}

int a2a_launch(const LaunchArgs &a) {
  return comm_all_to_all(a.comm, a.ptrs[0], a.ptrs[1], (size_t)a.step->ints[0], (int)a.step->ints[1], a.stream);
}

}  // namespace idx

NKB_REGISTER_KERNEL("alltoall", idx::a2a_launch, idx::coll_check);
NKB_REGISTER_KERNEL("allgather", idx::ag_launch, idx::coll_check);
NKB_REGISTER_KERNEL("reducescatter", idx::rs_launch, idx::coll_check);
NKB_REGISTER_KERNEL("take", idx::take_launch, idx::take_check);
NKB_REGISTER_KERNEL("gather_pts", idx::pts_launch, idx::pts_check);
NKB_REGISTER_KERNEL("pad", idx::pad_launch, idx::pad_check);
NKB_REGISTER_KERNEL("scatter_rows", idx::srows_launch, idx::srows_check);
NKB_REGISTER_KERNEL("scatter_pts", idx::spts_launch, idx::spts_check);
NKB_REGISTER_KERNEL("copy_bytes", idx::copy_launch, idx::copy_check);
NKB_REGISTER_KERNEL("allreduce", idx::ar_launch, idx::ar_check);
NKB_REGISTER_KERNEL("allreduce_add", idx::ara_launch, idx::ara_check);

}  // namespace nkb
