// All-reduce (sum) over NVLink SHARP: the HLO all-reduce of NKIPy's
// collectives (reference distributed/collectives.py:87-110) on B200s joined by
// NVSwitch, reduced inside the switch.
//
// Every rank holds the same symmetric region (a PyTorch symmetric-memory
// allocation bound to the communicator): a data area that is also mapped
// through an NVLink multicast object, and a flags area at its end.  The plan
// places the partial sum in the data area (its producer writes it there), and
// the reduction runs in place.  The payload of N bytes is viewed as `world`
// slices; CTA c of every rank owns sub-chunk c of every slice:
//   1. barrier with CTA c of every peer (sys-scope release/acquire flags):
//      every rank's partial is complete;
//   2. multimem.ld_reduce of sub-chunk c of this rank's slice (the switch
//      reads it from all GPUs and adds, accumulating in fp32), multimem.st of
//      the sum (the switch writes it to all GPUs);
//   3. barrier with CTA c of every peer: sub-chunk c of every slice holds the sum;
//   4. optionally, dst = residual + sum for sub-chunk c of every slice (the
//      add that follows a row-parallel block), so the sum is read once.
// Each GPU sends and receives about N(1 + 1/world) bytes over NVLink, against
// 2N(world-1)/world for a ring.  Barrier epochs are per-CTA counters in
// device memory, so the kernel replays inside CUDA graphs.  Every wait is
// bounded: on expiry the kernel records an error flag and returns.

#include "common.cuh"

namespace nkb {
namespace nvls {

constexpr int MAX_CTAS = 256, MAX_WORLD = 16, THREADS = 512;

__device__ int g_error = 0;

struct Args {
  const uint8_t *res;       // residual added to the sum (or null: the sum stays in `local`)
  uint8_t *dst;             // destination of residual + sum
  uint8_t *local;           // the payload in this rank's symmetric data area
  uint64_t mc;              // the same payload through the multicast object
  uint32_t *flags;          // this rank's flags [2][MAX_CTAS][MAX_WORLD]
  uint32_t *const *peer_flags;  // device array: each rank's flags, as mapped here
  uint32_t *epochs;         // [MAX_CTAS] per-CTA launch counters (device memory)
  size_t slice;             // bytes per slice (multiple of 16)
  int rank, world, f32;
  long long wait;           // budget of each barrier wait (SM clock cycles)
};

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// sum over all ranks of 16 bytes at a multicast address (read and added inside the switch)
__device__ __forceinline__ void ld_reduce(uint64_t addr, int f32, uint32_t *r) {
  if (f32)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "l"(addr));
  else
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "l"(addr));
}
// 16 bytes to every rank's copy of a multicast address
__device__ __forceinline__ void st_multi(uint64_t addr, const uint32_t *r) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// CTA c meets CTA c of every rank; false when the wait budget ran out
__device__ bool barrier(const Args &a, int phase, uint32_t epoch) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int t = threadIdx.x;
  if (t < a.world) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const size_t slot = ((size_t)phase * MAX_CTAS + blockIdx.x) * MAX_WORLD;
    st_release(a.peer_flags[t] + slot + a.rank, epoch);
    if (!wait_counter_geq(a.flags + slot + t, epoch, a.wait, nullptr, 0)) {
      atomicExch(&g_error, 1);
      ok = 0;
    }
  }
  __syncthreads();
  return ok != 0;
}

// dst = res + sum on 16 bytes (bf16 pairs or fp32), each sum rounded to the type
__device__ __forceinline__ uint4 add16(uint4 a, uint4 b, int f32) {
  uint32_t *x = reinterpret_cast<uint32_t *>(&a);
  const uint32_t *y = reinterpret_cast<const uint32_t *>(&b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (f32) {
      x[i] = __float_as_uint(__uint_as_float(x[i]) + __uint_as_float(y[i]));
    } else {
      const float2 p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&x[i]));
      const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&y[i]));
      const __nv_bfloat162 r = __floats2bfloat162_rn(p.x + q.x, p.y + q.y);
      x[i] = *reinterpret_cast<const uint32_t *>(&r);
    }
  }
  return a;
}

__global__ void __launch_bounds__(THREADS) nvls_allreduce_kernel(const __grid_constant__ Args a) {
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) epoch_s = ++a.epochs[blockIdx.x];
  __syncthreads();
  const uint32_t epoch = epoch_s;
  // this CTA's byte range inside each slice
  const size_t nvec = a.slice / 16;
  const size_t lo = nvec * blockIdx.x / gridDim.x * 16, hi = nvec * (blockIdx.x + 1) / gridDim.x * 16;

  if (!barrier(a, 0, epoch)) return;
  const uint64_t mine = a.mc + (uint64_t)a.rank * a.slice;
  // U independent reductions in flight per thread: each is a round trip through the switch
  constexpr int U = 4;
  const size_t step = (size_t)THREADS * 16;
  size_t o = lo + (size_t)threadIdx.x * 16;
  for (; o + (U - 1) * step < hi; o += U * step) {
    uint32_t r[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) ld_reduce(mine + o + u * step, a.f32, r[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) st_multi(mine + o + u * step, r[u]);
  }
  for (; o < hi; o += step) {
    uint32_t r[4];
    ld_reduce(mine + o, a.f32, r);
    st_multi(mine + o, r);
  }
  if (!barrier(a, 1, epoch)) return;
  if (a.res) {
    for (int s = 0; s < a.world; ++s) {
      const size_t base = (size_t)s * a.slice;
      for (size_t q = lo + (size_t)threadIdx.x * 16; q < hi; q += step)
        *reinterpret_cast<uint4 *>(a.dst + base + q) =
            add16(*reinterpret_cast<const uint4 *>(a.res + base + q), *reinterpret_cast<const uint4 *>(a.local + base + q),
                  a.f32);
    }
  }
}

// out = a + b elementwise (bf16 or fp32), 16 bytes per thread step; n16 = bytes / 16
__global__ void add_kernel(const uint4 *a, const uint4 *b, uint4 *out, size_t n16, int f32) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
    out[i] = add16(a[i], b[i], f32);
}

}  // namespace nvls

// Bytes of the flags area at the end of a bound symmetric region.
size_t nvls_flag_bytes() { return (size_t)2 * nvls::MAX_CTAS * nvls::MAX_WORLD * sizeof(uint32_t); }

// Can the NVLS path take this all-reduce?  (sum of bf16 or fp32 in place in
// the bound data area, slices of whole 16-byte vectors)
bool nvls_eligible(size_t count, int dtype, int world) {
  if (dtype != NKB_BF16 && dtype != NKB_F32) return false;
  if (world < 2 || world > nvls::MAX_WORLD) return false;
  const size_t bytes = count * dtype_size(dtype);
  return bytes > 0 && bytes % ((size_t)world * 16) == 0;
}

// buf: the payload inside this rank's symmetric data area; mc_buf: the same
// payload through the multicast object; res/dst: optional residual add
int nvls_all_reduce(void *buf, void *mc_buf, const void *res, void *dst, size_t count, int dtype, uint32_t *flags,
                    uint32_t *const *peer_flags, uint32_t *epochs, int rank, int world, int device,
                    cudaStream_t stream) {
  nvls::Args a;
  a.res = static_cast<const uint8_t *>(res);
  a.dst = static_cast<uint8_t *>(dst);
  a.local = static_cast<uint8_t *>(buf);
  a.mc = reinterpret_cast<uint64_t>(mc_buf);
  a.flags = flags;
  a.peer_flags = peer_flags;
  a.epochs = epochs;
  a.slice = count * dtype_size(dtype) / world;
  a.rank = rank;
  a.world = world;
  a.wait = wait_limit_cycles();
  a.f32 = dtype == NKB_F32;
  if (res && ((reinterpret_cast<uintptr_t>(res) | reinterpret_cast<uintptr_t>(dst)) & 15))
    return fail(NKB_ERR_UNSUPPORTED, "all-reduce + add: residual and destination must be 16-byte aligned");
  const size_t bytes_per_pass = 16 * nvls::THREADS;
  int ctas = (int)std::min<size_t>((a.slice + bytes_per_pass - 1) / bytes_per_pass, (size_t)num_sms(device));
  ctas = std::max(1, std::min(ctas, nvls::MAX_CTAS));
  nvls::nvls_allreduce_kernel<<<ctas, nvls::THREADS, 0, stream>>>(a);
  return launch_status("nvls_allreduce_kernel");
}

// out = a + b (bf16 or fp32, 16-byte aligned, bytes a multiple of 16; else a plain loop on the host side refuses)
int add_elementwise(const void *a, const void *b, void *out, size_t count, int dtype, cudaStream_t stream) {
  const size_t bytes = count * dtype_size(dtype);
  if ((dtype != NKB_BF16 && dtype != NKB_F32) || bytes % 16 ||
      ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out)) & 15))
    return fail(NKB_ERR_UNSUPPORTED, "all-reduce + add: bf16/fp32, 16-byte aligned, whole 16-byte vectors");
  if (!bytes) return NKB_OK;
  const size_t n16 = bytes / 16;
  const int grid = (int)std::min<size_t>((n16 + 255) / 256, 148 * 8);
  nvls::add_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4 *>(a), static_cast<const uint4 *>(b),
                                             static_cast<uint4 *>(out), n16, dtype == NKB_F32);
  return launch_status("add_kernel");
}

int nvls_read_and_clear_error(int *flag) {
  int zero = 0;
  NKB_CUDA_TRY(cudaMemcpyFromSymbol(flag, nvls::g_error, sizeof(int)));
  if (*flag) NKB_CUDA_TRY(cudaMemcpyToSymbol(nvls::g_error, &zero, sizeof(int)));
  return NKB_OK;
}

}  // namespace nkb
