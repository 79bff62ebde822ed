// Shared definitions of libnkb: error state, dtype helpers, the launch-step
// record that plans are decoded into, and the kernel registry.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>
#include <string>
#include <vector>

#include "../../include/nkb.h"

namespace nkb {

// ---- error reporting ------------------------------------------------------
void set_error(const std::string &msg);
int fail(int status, const std::string &msg);

#define NKB_CUDA_TRY(expr)                                                              \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess)                                                              \
      return ::nkb::fail(NKB_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define NKB_CHECK(cond, status, msg)       \
  do {                                     \
    if (!(cond)) return ::nkb::fail(status, msg); \
  } while (0)

// ---- dtypes -----------------------------------------------------------------
inline int dtype_size(int dt) {
  switch (dt) {
    case NKB_F32: case NKB_I32: case NKB_U32: return 4;
    case NKB_BF16: case NKB_F16: case NKB_I16: case NKB_U16: return 2;
    case NKB_I8: case NKB_U8: case NKB_BOOL: case NKB_F8E4M3: case NKB_F8E5M2: return 1;
    default: return 0;
  }
}
__host__ __device__ inline bool dtype_is_float(int dt) {
  return dt == NKB_F32 || dt == NKB_BF16 || dt == NKB_F16 || dt == NKB_F8E4M3 || dt == NKB_F8E5M2;
}

// Load one element of storage type `dt` at p[i] as raw 32-bit register bits:
// float dtypes widen to an fp32 bit pattern, integers to int32, bool to 0/1.
__device__ __forceinline__ uint32_t load_as_reg(const void *p, int64_t i, int dt) {
  switch (dt) {
    case NKB_F32: return __float_as_uint(static_cast<const float *>(p)[i]);
    case NKB_BF16: return __float_as_uint(__bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]));
    case NKB_F16: return __float_as_uint(__half2float(static_cast<const __half *>(p)[i]));
    case NKB_I32: case NKB_U32: return static_cast<const uint32_t *>(p)[i];
    case NKB_I16: return static_cast<uint32_t>(static_cast<int32_t>(static_cast<const int16_t *>(p)[i]));
    case NKB_U16: return static_cast<const uint16_t *>(p)[i];
    case NKB_I8: return static_cast<uint32_t>(static_cast<int32_t>(static_cast<const int8_t *>(p)[i]));
    case NKB_U8: return static_cast<const uint8_t *>(p)[i];
    case NKB_BOOL: return static_cast<const uint8_t *>(p)[i] ? 1u : 0u;
    default: return 0u;
  }
}

// One element of storage type `dt` at p[i] as an fp32 value (integers and
// bools converted by value: a product of mixed integer and float operands
// computes in fp32, as the traced dot's result type says).
__device__ __forceinline__ float load_as_float(const void *p, int64_t i, int dt) {
  const uint32_t r = load_as_reg(p, i, dt);
  switch (dt) {
    case NKB_I32: case NKB_I16: case NKB_I8: return (float)(int32_t)r;
    case NKB_U32: case NKB_U16: case NKB_U8: case NKB_BOOL: return (float)r;
    default: return __uint_as_float(r);
  }
}

__device__ __forceinline__ void store_from_reg(void *p, int64_t i, int dt, uint32_t v) {
  switch (dt) {
    case NKB_F32: static_cast<float *>(p)[i] = __uint_as_float(v); break;
    case NKB_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(__uint_as_float(v)); break;
    case NKB_F16: static_cast<__half *>(p)[i] = __float2half_rn(__uint_as_float(v)); break;
    case NKB_I32: case NKB_U32: static_cast<uint32_t *>(p)[i] = v; break;
    case NKB_I16: case NKB_U16: static_cast<uint16_t *>(p)[i] = static_cast<uint16_t>(v); break;
    case NKB_I8: case NKB_U8: static_cast<uint8_t *>(p)[i] = static_cast<uint8_t>(v); break;
    case NKB_BOOL: static_cast<uint8_t *>(p)[i] = v ? 1 : 0; break;
    default: break;
  }
}

// ---- launch steps -------------------------------------------------------------
// One kernel launch of a plan, after buffer resolution: device pointers (with
// byte offsets applied), integer and float parameters, and the stream.
struct Step {
  std::string kernel;
  std::vector<int> buf_ids;        // plan buffer id per pointer argument
  std::vector<int64_t> buf_offsets;  // byte offset inside that buffer
  std::vector<int64_t> ints;
  std::vector<float> floats;
};

struct LaunchArgs {
  const Step *step;
  void *const *ptrs;  // resolved device pointers, one per buf_ids entry
  cudaStream_t stream;
  void *comm;         // bound NCCL communicator (collective steps only)
  int device;
  // the launch may overlap the previous kernel on the stream (programmatic
  // dependent launch): false for the first step of an execute, which must
  // follow whatever ran on the stream before it in full
  bool pdl = false;
};

using LaunchFn = int (*)(const LaunchArgs &);
// Validation at plan load: returns NKB_OK or fails with a message.
using CheckFn = int (*)(const Step &);

struct KernelEntry {
  const char *name;
  LaunchFn launch;
  CheckFn check;
};

// Registry filled by each kernel translation unit (static initialisers).
void register_kernel(const char *name, LaunchFn fn, CheckFn check);
const KernelEntry *find_kernel(const std::string &name);

struct Registrar {
  Registrar(const char *name, LaunchFn fn, CheckFn check) { register_kernel(name, fn, check); }
};

#define NKB_CAT2(a, b) a##b
#define NKB_CAT(a, b) NKB_CAT2(a, b)
#define NKB_REGISTER_KERNEL(name, fn, check) \
  static ::nkb::Registrar NKB_CAT(_nkb_reg_, __LINE__)(name, fn, check)

// Kernel launch error check (kernel launches report via cudaGetLastError).
inline int launch_status(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NKB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return NKB_OK;
}

int num_sms(int device);

// Programmatic dependent launch.  A kernel started by launch_pdl may begin
// while the kernel before it on the stream is still draining (inside a CUDA
// graph the edge between the two becomes a programmatic one), so its launch
// and set-up overlap that kernel's tail.  Such a kernel calls pdl_wait()
// before its first global read or write (it returns once every earlier
// kernel on the stream has finished and its writes are visible), then
// pdl_trigger() so that the next kernel can be launched in turn.  Both are
// no-ops for a kernel started without the attribute, which launch_pdl gives
// only when `pdl` is true and NKB_PDL is not 0.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
bool pdl_enabled();
template <class... KArgs, class... Args>
cudaError_t launch_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Budget, in SM clock cycles, of the waits on counters that other ranks or
// other CTAs advance (the fused GEMM + all-reduce, the in-switch all-reduce
// barrier): set with nkb_set_wait_limit_us, 1 s by default.  Kernels receive
// it in their launch arguments.
long long wait_limit_cycles();

// Polls a counter (sys-scope acquire) until it reaches `target` (wrapping
// compare); false when `limit` cycles passed or *abort became nonzero first.
// `sleep_ns` > 0 lets the thread sleep between polls.
__device__ __forceinline__ bool wait_counter_geq(const uint32_t *p, uint32_t target, long long limit,
                                                 volatile int *abort, unsigned sleep_ns) {
  auto value = [p]() {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
  };
  if ((int)(value() - target) >= 0) return true;
  const long long t0 = clock64();
  while ((int)(value() - target) < 0) {
    if ((abort && *abort) || clock64() - t0 > limit) return false;
    if (sleep_ns) __nanosleep(sleep_ns);
  }
  return true;
}

// Id of the calling thread's current CUDA context (0 when there is none).
// A context created after a cudaDeviceReset gets a new id, and the kernels'
// module is loaded into it afresh.
unsigned long long context_id();

// One-time set-up per (device, CUDA context), e.g. a kernel's
// cudaFuncSetAttribute: thread-safe, and repeated after the device's context
// was reset, since the attribute belonged to the module of the old context.
class ContextOnce {
 public:
  template <class F>
  int run(int device, F &&set) {
    const unsigned long long id = context_id();
    if (device < 0 || device >= 64 || id == 0) return set();
    std::lock_guard<std::mutex> lk(mu_);
    if (done_[device] == id) return NKB_OK;
    if (int s = set()) return s;
    done_[device] = id;
    return NKB_OK;
  }

 private:
  std::mutex mu_;
  unsigned long long done_[64] = {};
};

// NCCL all-reduce entry (implemented in the runtime, which owns the dlopen).
int comm_all_reduce(void *comm, const void *src, void *dst, size_t count, int dtype, cudaStream_t stream);
// Fused GEMM + all-reduce: per-step flag slots after the all-reduce flags at
// the end of the bound symmetric region.  A slot holds SYMM_AR_CHUNKS arrival
// counts (one per 128-row block of the output), then a count of this rank's
// finished CTAs and a count of finished ranks.
constexpr int SYMM_AR_SLOTS = 4, SYMM_AR_CHUNKS = 1022, SYMM_AR_SLOT_BYTES = 4096;
struct SymmAr {
  uint64_t mc_payload;  // the payload through the multicast object
  uint32_t *flags;      // this rank's slot
  uint64_t mc_flags;    // the slot through the multicast object
  int rank, world;
};
// Fills `out` when `payload` (bytes) lies in the communicator's bound
// symmetric data area (16-byte aligned) and slot is valid; false otherwise.
bool comm_symm_ar(void *comm, const void *payload, size_t bytes, int slot, SymmAr *out);

// NCCL all-gather (recv = world * count, rank-major) and sum reduce-scatter
// (send = world * count); count is per rank.
int comm_all_gather(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream);
int comm_reduce_scatter(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream);
// all-to-all of (world, count) rank-major blocks (count per block)
int comm_all_to_all(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream);

// dst = res + all-reduce(buf) (buf keeps the sum)
int comm_all_reduce_add(void *comm, void *buf, const void *res, void *dst, size_t count, int dtype,
                        cudaStream_t stream);

}  // namespace nkb
