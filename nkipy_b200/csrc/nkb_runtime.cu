// libnkb runtime: the C ABI of include/nkb.h.
//
// Replaces Spike's C++ core (spike/src/spike.cpp, tensor.cpp, model.cpp,
// nrt_wrapper.cpp, sys_trace.cpp of shaojiex-aws/nkipy) with a CUDA runtime:
// one context per device, a default non-blocking stream, device buffers with
// bounds-checked copies, text launch plans decoded once at load, and an
// executor that issues the plan's kernels in order (optionally replayed from a
// captured CUDA graph).  NCCL is loaded with dlopen so the library has no
// link-time dependency on a particular NCCL build.

#include <cuda.h>
#include <dlfcn.h>
#include <nvtx3/nvToolsExt.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

// ---------------------------------------------------------------------------
// error state and registry
// ---------------------------------------------------------------------------
namespace nkb {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

int fail(int status, const std::string &msg) {
  g_last_error = msg;
  return status;
}

static std::vector<KernelEntry> &registry() {
  static std::vector<KernelEntry> r;
  return r;
}

void register_kernel(const char *name, LaunchFn fn, CheckFn check) {
  registry().push_back(KernelEntry{name, fn, check});
}

const KernelEntry *find_kernel(const std::string &name) {
  for (const auto &e : registry())
    if (name == e.name) return &e;
  return nullptr;
}

// Driver entry points resolved through the runtime (libnkb links no driver
// symbol directly, so it loads on machines without a driver).
unsigned long long context_id() {
  using GetCurrent = CUresult (*)(CUcontext *);
  using GetId = CUresult (*)(CUcontext, unsigned long long *);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cached[device]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cached[device] = v;
  }
  return cached[device];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("NKB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace nkb

using nkb::fail;

// ---------------------------------------------------------------------------
// runtime state
// ---------------------------------------------------------------------------
namespace {

struct RuntimeState {
  bool initialised = false;
  int device = 0;
  cudaStream_t stream = nullptr;
};

RuntimeState g_rt;
std::mutex g_mu;

}  // namespace

struct nkb_buf_s {
  uint32_t magic;
  void *ptr;
  size_t bytes;
  int device;
  bool owned;
  nkb_buf_s *parent;
  int refs;  // owner: 1 + live slices
};

namespace {
constexpr uint32_t kBufMagic = 0x4e4b4242;  // "NKBB"
std::set<nkb_buf_s *> g_live_bufs;

bool buf_ok(nkb_buf b) {
  std::lock_guard<std::mutex> lk(g_mu);
  return b && g_live_bufs.count(b) && b->magic == kBufMagic;
}

int ensure_init() {
  if (!g_rt.initialised) return fail(NKB_ERR_STATE, "nkb runtime not initialised (call nkb_init)");
  return NKB_OK;
}

void release_owner(nkb_buf_s *o) {
  if (--o->refs == 0) {
    if (o->owned && o->ptr) cudaFree(o->ptr);
    o->magic = 0;
    delete o;
  }
}
}  // namespace

// ---------------------------------------------------------------------------
// runtime
// ---------------------------------------------------------------------------
extern "C" int nkb_init(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(NKB_ERR_CUDA, std::string("no CUDA device visible: ") + cudaGetErrorString(e));
  if (device < 0 || device >= n) return fail(NKB_ERR_INVALID, "device index out of range");
  if (g_rt.initialised && g_rt.device == device) return NKB_OK;
  if (g_rt.initialised && g_rt.device != device)
    return fail(NKB_ERR_STATE, "nkb runtime already initialised on another device; call nkb_shutdown first");
  NKB_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  NKB_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10)
    return fail(NKB_ERR_UNSUPPORTED, std::string("libnkb is built for sm_100a; device is ") + prop.name);
  NKB_CUDA_TRY(cudaStreamCreateWithFlags(&g_rt.stream, cudaStreamNonBlocking));
  g_rt.device = device;
  g_rt.initialised = true;
  return NKB_OK;
}

extern "C" int nkb_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_rt.initialised) return NKB_OK;
  cudaStreamSynchronize(g_rt.stream);
  cudaStreamDestroy(g_rt.stream);
  g_rt = RuntimeState();
  return NKB_OK;
}

extern "C" int nkb_device_count(int *count) {
  if (!count) return fail(NKB_ERR_INVALID, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  *count = (e == cudaSuccess) ? n : 0;
  if (e != cudaSuccess) cudaGetLastError();
  return NKB_OK;
}

extern "C" const char *nkb_last_error(void) { return nkb::g_last_error.c_str(); }

extern "C" const char *nkb_status_str(int status) {
  switch (status) {
    case NKB_OK: return "ok";
    case NKB_ERR_INVALID: return "invalid argument";
    case NKB_ERR_CUDA: return "CUDA error";
    case NKB_ERR_PLAN: return "plan error";
    case NKB_ERR_UNSUPPORTED: return "unsupported";
    case NKB_ERR_NCCL: return "NCCL error";
    case NKB_ERR_STATE: return "invalid state";
    case NKB_ERR_DEVICE: return "device-reported error";
    default: return "unknown status";
  }
}

extern "C" int nkb_version(int *major, int *minor) {
  if (major) *major = 0;
  if (minor) *minor = 1;
  return NKB_OK;
}

namespace nkb {
int gemm_read_and_clear_error(int *flag);
int linattn_read_and_clear_error(int *flag);
int nvls_read_and_clear_error(int *flag);
int fa_read_and_clear_error(int *flag);
int transpose_read_and_clear_error(int *flag);
int waits_read_and_clear_error(int *flag);
int wait_probe_launch(const uint32_t *counter, uint32_t target, cudaStream_t stream);
}

extern "C" int nkb_device_error(int *flag) {
  if (int s = ensure_init()) return s;
  if (!flag) return fail(NKB_ERR_INVALID, "flag is NULL");
  int g = 0, l = 0, n = 0, f = 0, t = 0;
  if (int s = nkb::gemm_read_and_clear_error(&g)) return s;
  if (int s = nkb::linattn_read_and_clear_error(&l)) return s;
  if (int s = nkb::nvls_read_and_clear_error(&n)) return s;
  if (int s = nkb::fa_read_and_clear_error(&f)) return s;
  if (int s = nkb::transpose_read_and_clear_error(&t)) return s;
  int w = 0;
  if (int s = nkb::waits_read_and_clear_error(&w)) return s;
  *flag = g | l | n | f | t | w;
  return NKB_OK;
}

extern "C" int nkb_wait_probe(const uint32_t *counter, uint32_t target, void *stream) {
  if (int s = ensure_init()) return s;
  return nkb::wait_probe_launch(counter, target, stream ? static_cast<cudaStream_t>(stream) : g_rt.stream);
}

extern "C" int nkb_synchronize(void) {
  if (int s = ensure_init()) return s;
  NKB_CUDA_TRY(cudaStreamSynchronize(g_rt.stream));
  return NKB_OK;
}

// ---------------------------------------------------------------------------
// buffers
// ---------------------------------------------------------------------------
extern "C" int nkb_alloc(size_t bytes, int device, nkb_buf *out) {
  if (int s = ensure_init()) return s;
  if (!out) return fail(NKB_ERR_INVALID, "out is NULL");
  if (device != g_rt.device) return fail(NKB_ERR_INVALID, "buffer device differs from the runtime device");
  void *p = nullptr;
  if (bytes) {
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NKB_ERR_CUDA, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
  }
  auto *b = new nkb_buf_s{kBufMagic, p, bytes, device, true, nullptr, 1};
  std::lock_guard<std::mutex> lk(g_mu);
  g_live_bufs.insert(b);
  *out = b;
  return NKB_OK;
}

extern "C" int nkb_wrap(void *device_ptr, size_t bytes, int device, nkb_buf *out) {
  if (int s = ensure_init()) return s;
  if (!out || (!device_ptr && bytes)) return fail(NKB_ERR_INVALID, "bad wrap arguments");
  auto *b = new nkb_buf_s{kBufMagic, device_ptr, bytes, device, false, nullptr, 1};
  std::lock_guard<std::mutex> lk(g_mu);
  g_live_bufs.insert(b);
  *out = b;
  return NKB_OK;
}

extern "C" int nkb_slice(nkb_buf src, size_t offset, size_t bytes, nkb_buf *out) {
  if (!buf_ok(src)) return fail(NKB_ERR_STATE, "slice of an invalid or freed buffer");
  if (!out) return fail(NKB_ERR_INVALID, "out is NULL");
  if (bytes == 0) bytes = src->bytes > offset ? src->bytes - offset : 0;
  if (offset > src->bytes || bytes > src->bytes - offset)
    return fail(NKB_ERR_INVALID, "slice [" + std::to_string(offset) + ", +" + std::to_string(bytes) +
                                     ") exceeds buffer of " + std::to_string(src->bytes) + " bytes");
  nkb_buf_s *owner = src->parent ? src->parent : src;
  owner->refs++;
  auto *b = new nkb_buf_s{kBufMagic, static_cast<char *>(src->ptr) + offset, bytes, src->device, false, owner, 1};
  std::lock_guard<std::mutex> lk(g_mu);
  g_live_bufs.insert(b);
  *out = b;
  return NKB_OK;
}

extern "C" int nkb_free(nkb_buf buf) {
  if (!buf_ok(buf)) return fail(NKB_ERR_STATE, "free of an invalid or already freed buffer");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_live_bufs.erase(buf);
  }
  if (buf->parent) {
    nkb_buf_s *owner = buf->parent;
    buf->magic = 0;
    delete buf;
    release_owner(owner);
  } else {
    release_owner(buf);
  }
  return NKB_OK;
}

extern "C" int nkb_buf_info(nkb_buf buf, size_t *bytes, int *device, void **device_ptr) {
  if (!buf_ok(buf)) return fail(NKB_ERR_STATE, "invalid or freed buffer");
  if (bytes) *bytes = buf->bytes;
  if (device) *device = buf->device;
  if (device_ptr) *device_ptr = buf->ptr;
  return NKB_OK;
}

extern "C" int nkb_h2d(nkb_buf dst, const void *src, size_t bytes, size_t offset) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(dst)) return fail(NKB_ERR_STATE, "write to an invalid or freed buffer");
  if (offset > dst->bytes || bytes > dst->bytes - offset)
    return fail(NKB_ERR_INVALID, "write of " + std::to_string(bytes) + " bytes at offset " + std::to_string(offset) +
                                     " exceeds buffer of " + std::to_string(dst->bytes) + " bytes");
  if (!bytes) return NKB_OK;
  if (!src) return fail(NKB_ERR_INVALID, "source is NULL");
  NKB_CUDA_TRY(cudaMemcpyAsync(static_cast<char *>(dst->ptr) + offset, src, bytes, cudaMemcpyHostToDevice, g_rt.stream));
  NKB_CUDA_TRY(cudaStreamSynchronize(g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_d2h(nkb_buf src, void *dst, size_t bytes, size_t offset) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(src)) return fail(NKB_ERR_STATE, "read from an invalid or freed buffer");
  if (offset > src->bytes || bytes > src->bytes - offset)
    return fail(NKB_ERR_INVALID, "read of " + std::to_string(bytes) + " bytes at offset " + std::to_string(offset) +
                                     " exceeds buffer of " + std::to_string(src->bytes) + " bytes");
  if (!bytes) return NKB_OK;
  if (!dst) return fail(NKB_ERR_INVALID, "destination is NULL");
  NKB_CUDA_TRY(cudaMemcpyAsync(dst, static_cast<char *>(src->ptr) + offset, bytes, cudaMemcpyDeviceToHost, g_rt.stream));
  NKB_CUDA_TRY(cudaStreamSynchronize(g_rt.stream));
  return NKB_OK;
}

// ---- streams, events and asynchronous copies (pipelined callers) ----------
extern "C" int nkb_stream_create(void **stream) {
  if (int s = ensure_init()) return s;
  if (!stream) return fail(NKB_ERR_INVALID, "stream is NULL");
  cudaStream_t st = nullptr;
  NKB_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  *stream = st;
  return NKB_OK;
}

extern "C" int nkb_stream_destroy(void *stream) {
  if (int s = ensure_init()) return s;
  if (!stream) return fail(NKB_ERR_INVALID, "stream is NULL");
  NKB_CUDA_TRY(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return NKB_OK;
}

extern "C" int nkb_stream_synchronize(void *stream) {
  if (int s = ensure_init()) return s;
  NKB_CUDA_TRY(cudaStreamSynchronize(stream ? static_cast<cudaStream_t>(stream) : g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_event_create(void **event) {
  if (int s = ensure_init()) return s;
  if (!event) return fail(NKB_ERR_INVALID, "event is NULL");
  cudaEvent_t e = nullptr;
  NKB_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  *event = e;
  return NKB_OK;
}

extern "C" int nkb_event_destroy(void *event) {
  if (int s = ensure_init()) return s;
  if (!event) return fail(NKB_ERR_INVALID, "event is NULL");
  NKB_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return NKB_OK;
}

extern "C" int nkb_event_record(void *event, void *stream) {
  if (int s = ensure_init()) return s;
  if (!event) return fail(NKB_ERR_INVALID, "event is NULL");
  NKB_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), stream ? static_cast<cudaStream_t>(stream) : g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_stream_wait_event(void *stream, void *event) {
  if (int s = ensure_init()) return s;
  if (!event) return fail(NKB_ERR_INVALID, "event is NULL");
  NKB_CUDA_TRY(cudaStreamWaitEvent(stream ? static_cast<cudaStream_t>(stream) : g_rt.stream,
                                   static_cast<cudaEvent_t>(event), 0));
  return NKB_OK;
}

extern "C" int nkb_h2d_async(nkb_buf dst, const void *src, size_t bytes, size_t offset, void *stream) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(dst)) return fail(NKB_ERR_STATE, "write to an invalid or freed buffer");
  if (offset > dst->bytes || bytes > dst->bytes - offset)
    return fail(NKB_ERR_INVALID, "write of " + std::to_string(bytes) + " bytes at offset " + std::to_string(offset) +
                                     " exceeds buffer of " + std::to_string(dst->bytes) + " bytes");
  if (!bytes) return NKB_OK;
  if (!src) return fail(NKB_ERR_INVALID, "source is NULL");
  NKB_CUDA_TRY(cudaMemcpyAsync(static_cast<char *>(dst->ptr) + offset, src, bytes, cudaMemcpyHostToDevice,
                               stream ? static_cast<cudaStream_t>(stream) : g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_d2h_async(nkb_buf src, void *dst, size_t bytes, size_t offset, void *stream) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(src)) return fail(NKB_ERR_STATE, "read from an invalid or freed buffer");
  if (offset > src->bytes || bytes > src->bytes - offset)
    return fail(NKB_ERR_INVALID, "read of " + std::to_string(bytes) + " bytes at offset " + std::to_string(offset) +
                                     " exceeds buffer of " + std::to_string(src->bytes) + " bytes");
  if (!bytes) return NKB_OK;
  if (!dst) return fail(NKB_ERR_INVALID, "destination is NULL");
  NKB_CUDA_TRY(cudaMemcpyAsync(dst, static_cast<char *>(src->ptr) + offset, bytes, cudaMemcpyDeviceToHost,
                               stream ? static_cast<cudaStream_t>(stream) : g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_memset(nkb_buf dst, int value, size_t bytes, size_t offset) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(dst)) return fail(NKB_ERR_STATE, "memset of an invalid or freed buffer");
  if (offset > dst->bytes || bytes > dst->bytes - offset) return fail(NKB_ERR_INVALID, "memset out of bounds");
  NKB_CUDA_TRY(cudaMemsetAsync(static_cast<char *>(dst->ptr) + offset, value, bytes, g_rt.stream));
  return NKB_OK;
}

extern "C" int nkb_copy(nkb_buf dst, size_t dst_offset, nkb_buf src, size_t src_offset, size_t bytes) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(dst) || !buf_ok(src)) return fail(NKB_ERR_STATE, "copy with an invalid or freed buffer");
  if (dst_offset > dst->bytes || bytes > dst->bytes - dst_offset || src_offset > src->bytes ||
      bytes > src->bytes - src_offset)
    return fail(NKB_ERR_INVALID, "copy out of bounds");
  if (!bytes) return NKB_OK;
  NKB_CUDA_TRY(cudaMemcpyAsync(static_cast<char *>(dst->ptr) + dst_offset, static_cast<char *>(src->ptr) + src_offset,
                               bytes, cudaMemcpyDeviceToDevice, g_rt.stream));
  NKB_CUDA_TRY(cudaStreamSynchronize(g_rt.stream));
  return NKB_OK;
}

// ---------------------------------------------------------------------------
// NCCL (dlopen)
// ---------------------------------------------------------------------------
namespace {

typedef int ncclResult_t_;
typedef void *ncclComm_t_;
struct ncclUniqueId_ {
  char internal[NKB_COMM_ID_BYTES];
};

struct NcclApi {
  void *handle = nullptr;
  ncclResult_t_ (*GetUniqueId)(ncclUniqueId_ *) = nullptr;
  ncclResult_t_ (*CommInitRank)(ncclComm_t_ *, int, ncclUniqueId_, int) = nullptr;
  ncclResult_t_ (*CommDestroy)(ncclComm_t_) = nullptr;
  ncclResult_t_ (*AllReduce)(const void *, void *, size_t, int, int, ncclComm_t_, cudaStream_t) = nullptr;
  ncclResult_t_ (*AllGather)(const void *, void *, size_t, int, ncclComm_t_, cudaStream_t) = nullptr;
  ncclResult_t_ (*ReduceScatter)(const void *, void *, size_t, int, int, ncclComm_t_, cudaStream_t) = nullptr;
  ncclResult_t_ (*Send)(const void *, size_t, int, int, ncclComm_t_, cudaStream_t) = nullptr;
  ncclResult_t_ (*Recv)(void *, size_t, int, int, ncclComm_t_, cudaStream_t) = nullptr;
  ncclResult_t_ (*GroupStart)() = nullptr;
  ncclResult_t_ (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t_) = nullptr;
  bool loaded = false;
};

NcclApi g_nccl;

int load_nccl() {
  if (g_nccl.loaded) return NKB_OK;
  const char *names[] = {getenv("NKB_NCCL_LIBRARY"), "libnccl.so.2", "libnccl.so"};
  for (const char *n : names) {
    if (!n) continue;
    g_nccl.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (g_nccl.handle) break;
  }
  if (!g_nccl.handle) return fail(NKB_ERR_NCCL, std::string("cannot dlopen NCCL: ") + dlerror());
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(dlsym(g_nccl.handle, "ncclGetUniqueId"));
  g_nccl.CommInitRank = reinterpret_cast<decltype(g_nccl.CommInitRank)>(dlsym(g_nccl.handle, "ncclCommInitRank"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(dlsym(g_nccl.handle, "ncclCommDestroy"));
  g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(dlsym(g_nccl.handle, "ncclAllReduce"));
  g_nccl.GetErrorString = reinterpret_cast<decltype(g_nccl.GetErrorString)>(dlsym(g_nccl.handle, "ncclGetErrorString"));
  g_nccl.AllGather = reinterpret_cast<decltype(g_nccl.AllGather)>(dlsym(g_nccl.handle, "ncclAllGather"));
  g_nccl.ReduceScatter = reinterpret_cast<decltype(g_nccl.ReduceScatter)>(dlsym(g_nccl.handle, "ncclReduceScatter"));
  g_nccl.Send = reinterpret_cast<decltype(g_nccl.Send)>(dlsym(g_nccl.handle, "ncclSend"));
  g_nccl.Recv = reinterpret_cast<decltype(g_nccl.Recv)>(dlsym(g_nccl.handle, "ncclRecv"));
  g_nccl.GroupStart = reinterpret_cast<decltype(g_nccl.GroupStart)>(dlsym(g_nccl.handle, "ncclGroupStart"));
  g_nccl.GroupEnd = reinterpret_cast<decltype(g_nccl.GroupEnd)>(dlsym(g_nccl.handle, "ncclGroupEnd"));
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRank || !g_nccl.CommDestroy || !g_nccl.AllReduce)
    return fail(NKB_ERR_NCCL, "NCCL library lacks required symbols");
  g_nccl.loaded = true;
  return NKB_OK;
}

int nccl_dtype(int dt) {
  // ncclDataType_t: int8=0 uint8=1 int32=2 uint32=3 int64=4 uint64=5 f16=6 f32=7 f64=8 bf16=9
  switch (dt) {
    case NKB_I8: return 0;
    case NKB_U8: case NKB_BOOL: return 1;
    case NKB_I32: return 2;
    case NKB_U32: return 3;
    case NKB_F16: return 6;
    case NKB_F32: return 7;
    case NKB_BF16: return 9;
    default: return -1;
  }
}

}  // namespace

namespace nkb {
size_t nvls_flag_bytes();
bool nvls_eligible(size_t count, int dtype, int world);
int nvls_all_reduce(void *buf, void *mc_buf, const void *res, void *dst, size_t count, int dtype, uint32_t *flags,
                    uint32_t *const *peer_flags, uint32_t *epochs, int rank, int world, int device,
                    cudaStream_t stream);
int add_elementwise(const void *a, const void *b, void *out, size_t count, int dtype, cudaStream_t stream);
}  // namespace nkb

struct nkb_comm_s {
  ncclComm_t_ comm;
  int rank, world, device;
  // symmetric region bound with nkb_comm_bind_symm (NVLS all-reduce); unset -> NCCL
  void *symm_local = nullptr, *symm_mc = nullptr;
  size_t symm_data = 0;                 // bytes of the data area (the flags follow it)
  uint32_t **symm_peer_flags = nullptr;  // device array [world]
  uint32_t *symm_epochs = nullptr;       // device array, per-CTA launch counters
  ~nkb_comm_s() {
    if (symm_peer_flags) cudaFree(symm_peer_flags);
    if (symm_epochs) cudaFree(symm_epochs);
  }
};

extern "C" int nkb_comm_unique_id(void *id_out) {
  if (!id_out) return fail(NKB_ERR_INVALID, "id_out is NULL");
  if (int s = load_nccl()) return s;
  ncclUniqueId_ id;
  int r = g_nccl.GetUniqueId(&id);
  if (r) return fail(NKB_ERR_NCCL, std::string("ncclGetUniqueId: ") + g_nccl.GetErrorString(r));
  memcpy(id_out, id.internal, NKB_COMM_ID_BYTES);
  return NKB_OK;
}

extern "C" int nkb_comm_init(const void *id, int rank, int world, int device, nkb_comm *out) {
  if (int s = ensure_init()) return s;
  if (!id || !out || world < 1 || rank < 0 || rank >= world) return fail(NKB_ERR_INVALID, "bad communicator arguments");
  if (int s = load_nccl()) return s;
  ncclUniqueId_ uid;
  memcpy(uid.internal, id, NKB_COMM_ID_BYTES);
  NKB_CUDA_TRY(cudaSetDevice(device));
  ncclComm_t_ c = nullptr;
  int r = g_nccl.CommInitRank(&c, world, uid, rank);
  if (r) return fail(NKB_ERR_NCCL, std::string("ncclCommInitRank: ") + g_nccl.GetErrorString(r));
  *out = new nkb_comm_s{c, rank, world, device};
  return NKB_OK;
}

// flags at the end of a bound region: the all-reduce barrier flags, then the
// fused GEMM + all-reduce slots
extern "C" size_t nkb_comm_symm_flag_bytes(void) {
  return nkb::nvls_flag_bytes() + (size_t)nkb::SYMM_AR_SLOTS * nkb::SYMM_AR_SLOT_BYTES;
}

extern "C" int nkb_comm_bind_symm(nkb_comm comm, void *local, void *multicast, void *const *peers, int n_peers,
                                  size_t bytes) {
  if (int s = ensure_init()) return s;
  if (!comm || !local || !multicast || !peers) return fail(NKB_ERR_INVALID, "NULL argument");
  if (n_peers != comm->world) return fail(NKB_ERR_INVALID, "one peer pointer per rank is needed");
  if (comm->world > 16) return fail(NKB_ERR_UNSUPPORTED, "symmetric all-reduce supports at most 16 ranks");
  const size_t fb = nkb_comm_symm_flag_bytes();
  if (bytes <= fb + 16) return fail(NKB_ERR_INVALID, "symmetric region too small");
  if ((reinterpret_cast<uintptr_t>(local) | reinterpret_cast<uintptr_t>(multicast) | bytes) & 15)
    return fail(NKB_ERR_INVALID, "symmetric region must be 16-byte aligned");
  const size_t data = (bytes - fb) & ~size_t(15);
  NKB_CUDA_TRY(cudaSetDevice(comm->device));
  std::vector<uint32_t *> pf(comm->world);
  for (int r = 0; r < comm->world; ++r) {
    if (!peers[r]) return fail(NKB_ERR_INVALID, "NULL peer pointer");
    pf[r] = reinterpret_cast<uint32_t *>(static_cast<char *>(peers[r]) + data);
  }
  if (!comm->symm_peer_flags) NKB_CUDA_TRY(cudaMalloc(&comm->symm_peer_flags, 16 * sizeof(uint32_t *)));
  if (!comm->symm_epochs) {
    NKB_CUDA_TRY(cudaMalloc(&comm->symm_epochs, 1024 * sizeof(uint32_t)));
    NKB_CUDA_TRY(cudaMemset(comm->symm_epochs, 0, 1024 * sizeof(uint32_t)));
  }
  NKB_CUDA_TRY(cudaMemcpy(comm->symm_peer_flags, pf.data(), pf.size() * sizeof(uint32_t *), cudaMemcpyHostToDevice));
  // this rank's flags start at zero; the caller synchronises the ranks before the first all-reduce
  NKB_CUDA_TRY(cudaMemset(static_cast<char *>(local) + data, 0, fb));
  NKB_CUDA_TRY(cudaDeviceSynchronize());
  comm->symm_local = local;
  comm->symm_mc = multicast;
  comm->symm_data = data;
  return NKB_OK;
}



extern "C" int nkb_comm_free(nkb_comm comm) {
  if (!comm) return NKB_OK;
  if (g_nccl.loaded && comm->comm) g_nccl.CommDestroy(comm->comm);
  delete comm;
  return NKB_OK;
}

namespace nkb {
// The payload lies inside the bound symmetric data area and can be reduced
// there inside NVSwitch.
static bool symm_payload(const nkb_comm_s *c, const void *p, size_t count, int dtype) {
  if (!c->symm_local || !nvls_eligible(count, dtype, c->world)) return false;
  const char *lo = static_cast<const char *>(c->symm_local), *q = static_cast<const char *>(p);
  const size_t bytes = count * dtype_size(dtype);
  return q >= lo && q + bytes <= lo + c->symm_data && ((q - lo) & 15) == 0;
}

bool comm_symm_ar(void *comm, const void *payload, size_t bytes, int slot, SymmAr *out) {
  const auto *c = static_cast<const nkb_comm_s *>(comm);
  if (!c || c->world < 2 || !c->symm_local || slot < 0 || slot >= SYMM_AR_SLOTS) return false;
  const char *lo = static_cast<const char *>(c->symm_local), *q = static_cast<const char *>(payload);
  if (q < lo || q + bytes > lo + c->symm_data || ((q - lo) & 15)) return false;
  const size_t flag_off = c->symm_data + nvls_flag_bytes() + (size_t)slot * SYMM_AR_SLOT_BYTES;
  out->mc_payload = reinterpret_cast<uint64_t>(static_cast<char *>(c->symm_mc) + (q - lo));
  out->flags = reinterpret_cast<uint32_t *>(static_cast<char *>(c->symm_local) + flag_off);
  out->mc_flags = reinterpret_cast<uint64_t>(static_cast<char *>(c->symm_mc) + flag_off);
  out->rank = c->rank;
  out->world = c->world;
  return true;
}

static int nvls_on(nkb_comm_s *c, void *buf, const void *res, void *dst, size_t count, int dtype, cudaStream_t stream) {
  const size_t off = static_cast<char *>(buf) - static_cast<char *>(c->symm_local);
  return nvls_all_reduce(buf, static_cast<char *>(c->symm_mc) + off, res, dst, count, dtype,
                         reinterpret_cast<uint32_t *>(static_cast<char *>(c->symm_local) + c->symm_data),
                         c->symm_peer_flags, c->symm_epochs, c->rank, c->world, c->device, stream);
}

int comm_all_reduce(void *comm, const void *src, void *dst, size_t count, int dtype, cudaStream_t stream) {
  auto *c = static_cast<nkb_comm_s *>(comm);
  if (!c) return fail(NKB_ERR_STATE, "all-reduce step but no communicator is bound to the plan");
  int nd = nccl_dtype(dtype);
  if (nd < 0) return fail(NKB_ERR_UNSUPPORTED, "dtype not supported by NCCL all-reduce");
  if (c->world == 1) {
    if (src != dst) NKB_CUDA_TRY(cudaMemcpyAsync(dst, src, count * dtype_size(dtype), cudaMemcpyDeviceToDevice, stream));
    return NKB_OK;
  }
  if (src == dst && symm_payload(c, dst, count, dtype)) return nvls_on(c, dst, nullptr, nullptr, count, dtype, stream);
  int r = g_nccl.AllReduce(src, dst, count, nd, /*ncclSum*/ 0, c->comm, stream);
  if (r) return fail(NKB_ERR_NCCL, std::string("ncclAllReduce: ") + g_nccl.GetErrorString(r));
  return NKB_OK;
}

// recv (world * count) = the ranks' send (count each), rank-major
int comm_all_gather(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream) {
  auto *c = static_cast<nkb_comm_s *>(comm);
  if (!c) return fail(NKB_ERR_STATE, "all-gather step but no communicator is bound to the plan");
  const size_t bytes = count * dtype_size(dtype);
  if (c->world == 1) {
    if (send != recv && bytes) NKB_CUDA_TRY(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream));
    return NKB_OK;
  }
  if (!g_nccl.AllGather) return fail(NKB_ERR_NCCL, "NCCL library lacks ncclAllGather");
  // NCCL takes bytes as uint8 so every dtype (bool, fp8 included) gathers
  int r = g_nccl.AllGather(send, recv, bytes, /*ncclUint8*/ 1, c->comm, stream);
  if (r) return fail(NKB_ERR_NCCL, std::string("ncclAllGather: ") + g_nccl.GetErrorString(r));
  return NKB_OK;
}

// recv (count) = sum over the ranks of their send block `rank` (send holds world * count)
int comm_reduce_scatter(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream) {
  auto *c = static_cast<nkb_comm_s *>(comm);
  if (!c) return fail(NKB_ERR_STATE, "reduce-scatter step but no communicator is bound to the plan");
  int nd = nccl_dtype(dtype);
  if (nd < 0) return fail(NKB_ERR_UNSUPPORTED, "dtype not supported by NCCL reduce-scatter");
  if (c->world == 1) {
    if (send != recv && count)
      NKB_CUDA_TRY(cudaMemcpyAsync(recv, send, count * dtype_size(dtype), cudaMemcpyDeviceToDevice, stream));
    return NKB_OK;
  }
  if (!g_nccl.ReduceScatter) return fail(NKB_ERR_NCCL, "NCCL library lacks ncclReduceScatter");
  int r = g_nccl.ReduceScatter(send, recv, count, nd, /*ncclSum*/ 0, c->comm, stream);
  if (r) return fail(NKB_ERR_NCCL, std::string("ncclReduceScatter: ") + g_nccl.GetErrorString(r));
  return NKB_OK;
}

// send and recv are (world, count) rank-major: block j of send goes to rank j,
// block i of recv comes from rank i
int comm_all_to_all(void *comm, const void *send, void *recv, size_t count, int dtype, cudaStream_t stream) {
  auto *c = static_cast<nkb_comm_s *>(comm);
  if (!c) return fail(NKB_ERR_STATE, "all-to-all step but no communicator is bound to the plan");
  const size_t bytes = count * dtype_size(dtype);
  if (c->world == 1) {
    if (send != recv && bytes) NKB_CUDA_TRY(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream));
    return NKB_OK;
  }
  if (!g_nccl.Send || !g_nccl.Recv || !g_nccl.GroupStart || !g_nccl.GroupEnd)
    return fail(NKB_ERR_NCCL, "NCCL library lacks point-to-point calls");
  int r = g_nccl.GroupStart();
  for (int p = 0; !r && p < c->world; ++p) {
    r = g_nccl.Send(static_cast<const char *>(send) + p * bytes, bytes, /*ncclUint8*/ 1, p, c->comm, stream);
    if (!r) r = g_nccl.Recv(static_cast<char *>(recv) + p * bytes, bytes, /*ncclUint8*/ 1, p, c->comm, stream);
  }
  int r2 = g_nccl.GroupEnd();
  if (r || r2) return fail(NKB_ERR_NCCL, std::string("all-to-all: ") + g_nccl.GetErrorString(r ? r : r2));
  return NKB_OK;
}

// dst = res + (sum over the ranks of buf); buf holds the sum afterwards
int comm_all_reduce_add(void *comm, void *buf, const void *res, void *dst, size_t count, int dtype,
                        cudaStream_t stream) {
  auto *c = static_cast<nkb_comm_s *>(comm);
  if (!c) return fail(NKB_ERR_STATE, "all-reduce step but no communicator is bound to the plan");
  if (c->world > 1 && symm_payload(c, buf, count, dtype)) return nvls_on(c, buf, res, dst, count, dtype, stream);
  if (int s = comm_all_reduce(comm, buf, buf, count, dtype, stream)) return s;
  return add_elementwise(res, buf, dst, count, dtype, stream);
}
}  // namespace nkb

extern "C" int nkb_comm_all_reduce(nkb_comm comm, nkb_buf buf, size_t count, int dtype, void *stream) {
  if (int s = ensure_init()) return s;
  if (!buf_ok(buf)) return fail(NKB_ERR_STATE, "invalid buffer");
  if (count * nkb::dtype_size(dtype) > buf->bytes) return fail(NKB_ERR_INVALID, "all-reduce count exceeds buffer");
  return nkb::comm_all_reduce(comm, buf->ptr, buf->ptr, count, dtype,
                              stream ? static_cast<cudaStream_t>(stream) : g_rt.stream);
}

extern "C" int nkb_comm_all_gather(nkb_comm comm, const void *send, void *recv, size_t count, int dtype,
                                   void *stream) {
  if (int s = ensure_init()) return s;
  if (!comm) return fail(NKB_ERR_STATE, "no communicator");
  return nkb::comm_all_gather(comm, send, recv, count, dtype, stream ? static_cast<cudaStream_t>(stream) : g_rt.stream);
}

extern "C" int nkb_comm_all_to_all(nkb_comm comm, const void *send, void *recv, size_t count, int dtype,
                                   void *stream) {
  if (int s = ensure_init()) return s;
  if (!comm) return fail(NKB_ERR_STATE, "no communicator");
  return nkb::comm_all_to_all(comm, send, recv, count, dtype, stream ? static_cast<cudaStream_t>(stream) : g_rt.stream);
}

extern "C" int nkb_comm_reduce_scatter(nkb_comm comm, const void *send, void *recv, size_t count, int dtype,
                                       void *stream) {
  if (int s = ensure_init()) return s;
  if (!comm) return fail(NKB_ERR_STATE, "no communicator");
  return nkb::comm_reduce_scatter(comm, send, recv, count, dtype,
                                  stream ? static_cast<cudaStream_t>(stream) : g_rt.stream);
}

// ---------------------------------------------------------------------------
// plans
// ---------------------------------------------------------------------------
namespace {

enum BufKind { BK_IN = 0, BK_OUT = 1, BK_CONST = 2, BK_TMP = 3, BK_SYMM = 4 };

struct PlanBuffer {
  BufKind kind;
  int index;        // io / const index
  size_t offset;    // arena offset (tmp) or offset in the symmetric region (symm)
  size_t bytes;
};

}  // namespace

struct nkb_plan_s {
  std::string name;
  int device = 0;
  std::vector<size_t> in_bytes, out_bytes, const_bytes;
  std::vector<void *> const_ptrs;
  size_t scratch = 0;
  void *arena = nullptr;
  size_t symm = 0;                // bytes of the symmetric region the plan's symm buffers need
  void *symm_fallback = nullptr;  // used for them while no large-enough region is bound
  std::vector<PlanBuffer> buffers;
  std::vector<nkb::Step> steps;
  std::vector<const nkb::KernelEntry *> entries;
  nkb_comm comm = nullptr;
  // graph replay cache: one instantiated graph per (io pointers, stream), a
  // few of them (alternating io buffer sets, as a pipelined caller binds)
  struct GraphEntry {
    std::vector<void *> key;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
  };
  static constexpr size_t kGraphCache = 4;
  std::vector<GraphEntry> graphs;
  uint64_t graph_clock = 0;
  int graph_kernels = -1;  // kernel nodes of the last captured graph (-1: none captured yet)
  // timing graph: the plan with an event record between every two steps (one
  // io binding, rebuilt when the binding changes)
  std::vector<void *> tkey;
  cudaGraphExec_t texec = nullptr;
  std::vector<cudaEvent_t> tev;
  ~nkb_plan_s() {
    for (auto &g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    if (texec) cudaGraphExecDestroy(texec);
    for (auto e : tev) cudaEventDestroy(e);
    for (void *p : const_ptrs)
      if (p) cudaFree(p);
    if (arena) cudaFree(arena);
    if (symm_fallback) cudaFree(symm_fallback);
  }
};

namespace {

int parse_plan(const std::string &text, nkb_plan_s *p) {
  std::istringstream in(text);
  std::string tok;
  in >> tok;
  if (tok != "NKBPLAN") return fail(NKB_ERR_PLAN, "plan text must start with NKBPLAN");
  int version = 0;
  in >> version;
  if (version != 1) return fail(NKB_ERR_PLAN, "unsupported plan version " + std::to_string(version));
  while (in >> tok) {
    if (tok == "end") return NKB_OK;
    if (tok == "name") {
      in >> p->name;
    } else if (tok == "inputs") {
      size_t n;
      in >> n;
      p->in_bytes.assign(n, 0);
    } else if (tok == "input" || tok == "output" || tok == "const") {
      size_t i, b;
      in >> i >> b;
      auto &v = tok == "input" ? p->in_bytes : tok == "output" ? p->out_bytes : p->const_bytes;
      if (i >= v.size()) return fail(NKB_ERR_PLAN, tok + " index out of range");
      v[i] = b;
    } else if (tok == "outputs") {
      size_t n;
      in >> n;
      p->out_bytes.assign(n, 0);
    } else if (tok == "consts") {
      size_t n;
      in >> n;
      p->const_bytes.assign(n, 0);
    } else if (tok == "scratch") {
      in >> p->scratch;
    } else if (tok == "symm") {
      in >> p->symm;

    } else if (tok == "buffers") {
      size_t n;
      in >> n;
      p->buffers.assign(n, PlanBuffer{BK_TMP, -1, 0, 0});
    } else if (tok == "buffer") {
      size_t id;
      std::string kind;
      in >> id >> kind;
      if (id >= p->buffers.size()) return fail(NKB_ERR_PLAN, "buffer id out of range");
      PlanBuffer &b = p->buffers[id];
      if (kind == "in" || kind == "out" || kind == "const") {
        in >> b.index;
        b.kind = kind == "in" ? BK_IN : kind == "out" ? BK_OUT : BK_CONST;
        const auto &v = b.kind == BK_IN ? p->in_bytes : b.kind == BK_OUT ? p->out_bytes : p->const_bytes;
        if (b.index < 0 || (size_t)b.index >= v.size()) return fail(NKB_ERR_PLAN, "buffer io index out of range");
        b.bytes = v[b.index];
      } else if (kind == "tmp") {
        b.kind = BK_TMP;
        in >> b.offset >> b.bytes;
        if (b.offset + b.bytes > p->scratch) return fail(NKB_ERR_PLAN, "tmp buffer exceeds scratch arena");
      } else if (kind == "symm") {
        b.kind = BK_SYMM;
        in >> b.offset >> b.bytes;
        if (b.offset + b.bytes > p->symm) return fail(NKB_ERR_PLAN, "symm buffer exceeds the plan's symmetric region");

      } else {
        return fail(NKB_ERR_PLAN, "unknown buffer kind " + kind);
      }
    } else if (tok == "steps") {
      size_t n;
      in >> n;
      p->steps.reserve(n);
    } else if (tok == "step") {
      nkb::Step s;
      int nb, ni, nf;
      in >> s.kernel >> nb;
      if (!in || nb < 0 || nb > 64) return fail(NKB_ERR_PLAN, "bad step header");
      for (int i = 0; i < nb; ++i) {
        int id;
        long long off;
        in >> id >> off;
        if (id < 0 || (size_t)id >= p->buffers.size()) return fail(NKB_ERR_PLAN, "step buffer id out of range");
        s.buf_ids.push_back(id);
        s.buf_offsets.push_back(off);
      }
      in >> ni;
      if (!in || ni < 0 || ni > 4096) return fail(NKB_ERR_PLAN, "bad step int count");
      for (int i = 0; i < ni; ++i) {
        long long v;
        in >> v;
        s.ints.push_back(v);
      }
      in >> nf;
      if (!in || nf < 0 || nf > 4096) return fail(NKB_ERR_PLAN, "bad step float count");
      for (int i = 0; i < nf; ++i) {
        std::string f;
        in >> f;
        s.floats.push_back(strtof(f.c_str(), nullptr));
      }
      if (!in) return fail(NKB_ERR_PLAN, "truncated step");
      p->steps.push_back(std::move(s));
    } else {
      return fail(NKB_ERR_PLAN, "unknown plan token '" + tok + "'");
    }
  }
  return fail(NKB_ERR_PLAN, "plan text has no 'end'");
}

}  // namespace

extern "C" int nkb_plan_load(const char *text, size_t len, int device, nkb_plan *out) {
  if (int s = ensure_init()) return s;
  if (!text || !out) return fail(NKB_ERR_INVALID, "NULL argument");
  auto p = std::make_unique<nkb_plan_s>();
  p->device = device;
  if (device != g_rt.device) return fail(NKB_ERR_INVALID, "plan device differs from the runtime's device");
  // the plan's device current on this thread: kernel checks below may load
  // modules (the elementwise chain compiler) into its context
  NKB_CUDA_TRY(cudaSetDevice(device));
  if (int s = parse_plan(std::string(text, len), p.get())) return s;
  for (const auto &st : p->steps) {
    const nkb::KernelEntry *e = nkb::find_kernel(st.kernel);
    if (!e) return fail(NKB_ERR_PLAN, "plan uses unknown kernel '" + st.kernel + "'");
    if (e->check) {
      if (int s = e->check(st)) return s;
    }
    for (size_t i = 0; i < st.buf_ids.size(); ++i) {
      const PlanBuffer &b = p->buffers[st.buf_ids[i]];
      if (st.buf_offsets[i] < 0 || (size_t)st.buf_offsets[i] > b.bytes)
        return fail(NKB_ERR_PLAN, "step '" + st.kernel + "' offset outside its buffer");
    }
    p->entries.push_back(e);
  }
  if (p->scratch) {
    cudaError_t e = cudaMalloc(&p->arena, p->scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NKB_ERR_CUDA, "scratch arena cudaMalloc(" + std::to_string(p->scratch) + "): " + cudaGetErrorString(e));
    }
  }
  p->const_ptrs.assign(p->const_bytes.size(), nullptr);
  for (size_t i = 0; i < p->const_bytes.size(); ++i) {
    if (!p->const_bytes[i]) continue;
    cudaError_t e = cudaMalloc(&p->const_ptrs[i], p->const_bytes[i]);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NKB_ERR_CUDA, std::string("constant cudaMalloc: ") + cudaGetErrorString(e));
    }
  }
  *out = p.release();
  return NKB_OK;
}

extern "C" int nkb_plan_free(nkb_plan plan) {
  if (!plan) return NKB_OK;
  cudaDeviceSynchronize();
  delete plan;
  return NKB_OK;
}

extern "C" int nkb_plan_num_io(nkb_plan plan, int *n_inputs, int *n_outputs) {
  if (!plan) return fail(NKB_ERR_INVALID, "NULL plan");
  if (n_inputs) *n_inputs = (int)plan->in_bytes.size();
  if (n_outputs) *n_outputs = (int)plan->out_bytes.size();
  return NKB_OK;
}

extern "C" int nkb_plan_io_bytes(nkb_plan plan, int is_output, int index, size_t *bytes) {
  if (!plan || !bytes) return fail(NKB_ERR_INVALID, "NULL argument");
  const auto &v = is_output ? plan->out_bytes : plan->in_bytes;
  if (index < 0 || (size_t)index >= v.size()) return fail(NKB_ERR_INVALID, "io index out of range");
  *bytes = v[index];
  return NKB_OK;
}

extern "C" int nkb_plan_num_consts(nkb_plan plan, int *n) {
  if (!plan || !n) return fail(NKB_ERR_INVALID, "NULL argument");
  *n = (int)plan->const_bytes.size();
  return NKB_OK;
}

extern "C" int nkb_plan_set_const(nkb_plan plan, int index, const void *host, size_t bytes) {
  if (int s = ensure_init()) return s;
  if (!plan || !host) return fail(NKB_ERR_INVALID, "NULL argument");
  if (index < 0 || (size_t)index >= plan->const_bytes.size()) return fail(NKB_ERR_INVALID, "const index out of range");
  if (bytes != plan->const_bytes[index])
    return fail(NKB_ERR_INVALID, "constant " + std::to_string(index) + " expects " +
                                     std::to_string(plan->const_bytes[index]) + " bytes, got " + std::to_string(bytes));
  NKB_CUDA_TRY(cudaMemcpy(plan->const_ptrs[index], host, bytes, cudaMemcpyHostToDevice));
  return NKB_OK;
}

extern "C" int nkb_plan_num_launches(nkb_plan plan, int *n) {
  if (!plan || !n) return fail(NKB_ERR_INVALID, "NULL argument");
  *n = (int)plan->steps.size();
  return NKB_OK;
}

extern "C" int nkb_plan_graph_kernels(nkb_plan plan, int *n) {
  if (!plan || !n) return fail(NKB_ERR_INVALID, "NULL argument");
  *n = plan->graph_kernels;
  return NKB_OK;
}

extern "C" int nkb_plan_scratch_bytes(nkb_plan plan, size_t *bytes) {
  if (!plan || !bytes) return fail(NKB_ERR_INVALID, "NULL argument");
  *bytes = plan->scratch;
  return NKB_OK;
}

extern "C" int nkb_plan_bind_comm(nkb_plan plan, nkb_comm comm) {
  if (!plan) return fail(NKB_ERR_INVALID, "NULL plan");
  plan->comm = comm;
  return NKB_OK;
}

namespace {

int resolve_io(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
               std::vector<void *> &base) {
  if (n_in != (int)plan->in_bytes.size() || n_out != (int)plan->out_bytes.size())
    return fail(NKB_ERR_INVALID, "plan '" + plan->name + "' expects " + std::to_string(plan->in_bytes.size()) +
                                     " inputs / " + std::to_string(plan->out_bytes.size()) + " outputs, got " +
                                     std::to_string(n_in) + " / " + std::to_string(n_out));
  base.assign(plan->buffers.size(), nullptr);
  for (size_t i = 0; i < plan->buffers.size(); ++i) {
    const PlanBuffer &b = plan->buffers[i];
    nkb_buf h = nullptr;
    switch (b.kind) {
      case BK_IN: h = ins[b.index]; break;
      case BK_OUT: h = outs[b.index]; break;
      case BK_CONST: base[i] = plan->const_ptrs[b.index]; continue;
      case BK_TMP: base[i] = static_cast<char *>(plan->arena) + b.offset; continue;
      case BK_SYMM: {
        // the communicator's symmetric region when one large enough is bound
        // (all-reduces then run inside NVSwitch), else a region of the plan's own
        nkb_comm c = plan->comm;
        if (c && c->symm_local && plan->symm <= c->symm_data) {
          base[i] = static_cast<char *>(c->symm_local) + b.offset;
        } else {
          if (!plan->symm_fallback) {
            cudaError_t e = cudaMalloc(&plan->symm_fallback, plan->symm);
            if (e != cudaSuccess) {
              cudaGetLastError();
              plan->symm_fallback = nullptr;
              return fail(NKB_ERR_CUDA, std::string("symm buffer cudaMalloc: ") + cudaGetErrorString(e));
            }
          }
          base[i] = static_cast<char *>(plan->symm_fallback) + b.offset;
        }
        continue;
      }
    }
    if (!buf_ok(h)) return fail(NKB_ERR_STATE, "plan io buffer " + std::to_string(i) + " is invalid or freed");
    if (h->bytes < b.bytes)
      return fail(NKB_ERR_INVALID, std::string(b.kind == BK_IN ? "input " : "output ") + std::to_string(b.index) +
                                       " has " + std::to_string(h->bytes) + " bytes, plan needs " +
                                       std::to_string(b.bytes));
    base[i] = h->ptr;
  }
  return NKB_OK;
}

int launch_steps(nkb_plan plan, const std::vector<void *> &base, cudaStream_t stream) {
  std::vector<void *> ptrs;
  for (size_t i = 0; i < plan->steps.size(); ++i) {
    const nkb::Step &st = plan->steps[i];
    ptrs.resize(st.buf_ids.size());
    for (size_t j = 0; j < st.buf_ids.size(); ++j)
      ptrs[j] = static_cast<char *>(base[st.buf_ids[j]]) + st.buf_offsets[j];
    nkb::LaunchArgs a{&st, ptrs.data(), stream, plan->comm ? (void *)plan->comm : nullptr, plan->device};
    a.pdl = i > 0;  // the first step follows earlier work on the stream in full
    // one NVTX range per launch, named after the kernel (seen by a profiler when one is attached)
    nvtxRangePushA(st.kernel.c_str());
    int s = plan->entries[i]->launch(a);
    nvtxRangePop();
    if (s) {
      std::string m = nkb_last_error();
      return fail(s, "step " + std::to_string(i) + " (" + st.kernel + "): " + m);
    }
  }
  return NKB_OK;
}

int execute_on(nkb_plan plan, const std::vector<void *> &base, cudaStream_t stream, bool use_graph) {
  if (!use_graph) return launch_steps(plan, base, stream);
  nkb_plan_s::GraphEntry *hit = nullptr;
  for (auto &g : plan->graphs)
    if (g.exec && g.stream == stream && g.key == base) hit = &g;
  if (!hit) {
    // a free slot, else the least recently used one
    if (plan->graphs.size() < nkb_plan_s::kGraphCache) {
      plan->graphs.emplace_back();
      hit = &plan->graphs.back();
    } else {
      hit = &plan->graphs[0];
      for (auto &g : plan->graphs)
        if (g.used < hit->used) hit = &g;
    }
    if (hit->exec) {
      cudaGraphExecDestroy(hit->exec);
      hit->exec = nullptr;
    }
    cudaGraph_t g = nullptr;
    NKB_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    int s = launch_steps(plan, base, stream);
    cudaError_t e = cudaStreamEndCapture(stream, &g);
    if (s) {
      if (g) cudaGraphDestroy(g);
      return s;
    }
    if (e != cudaSuccess) return fail(NKB_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    {
      // the kernels one execute launches (steps may launch none, one or two)
      size_t nn = 0;
      int kernels = 0;
      if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
        std::vector<cudaGraphNode_t> nodes(nn);
        if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
          for (auto nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
          }
      }
      plan->graph_kernels = kernels;
    }
    e = cudaGraphInstantiate(&hit->exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      hit->exec = nullptr;
      return fail(NKB_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    }
    hit->key = base;
    hit->stream = stream;
  }
  hit->used = ++plan->graph_clock;
  NKB_CUDA_TRY(cudaGraphLaunch(hit->exec, stream));
  return NKB_OK;
}

}  // namespace

extern "C" int nkb_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out, void *stream,
                           int use_graph) {
  if (int s = ensure_init()) return s;
  if (!plan) return fail(NKB_ERR_INVALID, "NULL plan");
  std::vector<void *> base;
  if (int s = resolve_io(plan, ins, n_in, outs, n_out, base)) return s;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g_rt.stream;
  return execute_on(plan, base, st, use_graph != 0);
}

extern "C" int nkb_time_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                                int warmup, int iters, int use_graph, float *ms_out) {
  if (int s = ensure_init()) return s;
  if (!plan || iters < 1 || !ms_out) return fail(NKB_ERR_INVALID, "bad timing arguments");
  std::vector<void *> base;
  if (int s = resolve_io(plan, ins, n_in, outs, n_out, base)) return s;
  cudaStream_t st = g_rt.stream;
  for (int i = 0; i < warmup; ++i)
    if (int s = execute_on(plan, base, st, use_graph != 0)) return s;
  std::vector<cudaEvent_t> ev(iters + 1);
  for (auto &e : ev) NKB_CUDA_TRY(cudaEventCreate(&e));
  int status = NKB_OK;
  cudaEventRecord(ev[0], st);
  for (int i = 0; i < iters && !status; ++i) {
    status = execute_on(plan, base, st, use_graph != 0);
    cudaEventRecord(ev[i + 1], st);
  }
  cudaError_t e = cudaStreamSynchronize(st);
  if (!status && e != cudaSuccess) status = fail(NKB_ERR_CUDA, std::string("timed execute: ") + cudaGetErrorString(e));
  if (!status)
    for (int i = 0; i < iters; ++i) cudaEventElapsedTime(&ms_out[i], ev[i], ev[i + 1]);
  for (auto &x : ev) cudaEventDestroy(x);
  return status;
}

// One graph replay of the plan with an event record node before the first
// step and after every step: the execute's time and each step's share of it,
// measured inside the replayed graph (steps keep their overlap with their
// neighbours; the event nodes add a few microseconds to the replay).
extern "C" int nkb_time_execute_steps(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                                      float *total_ms, float *step_ms) {
  if (int s = ensure_init()) return s;
  if (!plan || !total_ms || !step_ms) return fail(NKB_ERR_INVALID, "bad timing arguments");
  std::vector<void *> base;
  if (int s = resolve_io(plan, ins, n_in, outs, n_out, base)) return s;
  cudaStream_t st = g_rt.stream;
  const size_t n = plan->steps.size();
  if (!plan->texec || plan->tkey != base) {
    if (plan->texec) cudaGraphExecDestroy(plan->texec);
    plan->texec = nullptr;
    for (auto e : plan->tev) cudaEventDestroy(e);
    plan->tev.assign(n + 1, nullptr);
    for (auto &e : plan->tev) NKB_CUDA_TRY(cudaEventCreate(&e));
    std::vector<void *> ptrs;
    cudaGraph_t g = nullptr;
    NKB_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int status = NKB_OK;
    // external record nodes: the events are recorded when the graph runs (a plain
    // record under capture only orders work inside the graph)
    cudaEventRecordWithFlags(plan->tev[0], st, cudaEventRecordExternal);
    for (size_t i = 0; i < n && !status; ++i) {
      const nkb::Step &stp = plan->steps[i];
      ptrs.resize(stp.buf_ids.size());
      for (size_t j = 0; j < stp.buf_ids.size(); ++j)
        ptrs[j] = static_cast<char *>(base[stp.buf_ids[j]]) + stp.buf_offsets[j];
      nkb::LaunchArgs a{&stp, ptrs.data(), st, plan->comm ? (void *)plan->comm : nullptr, plan->device};
      a.pdl = false;  // an event node sits between every two launches
      status = plan->entries[i]->launch(a);
      cudaEventRecordWithFlags(plan->tev[i + 1], st, cudaEventRecordExternal);
    }
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (status) {
      if (g) cudaGraphDestroy(g);
      return status;
    }
    if (e != cudaSuccess) return fail(NKB_ERR_CUDA, std::string("timing graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&plan->texec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      plan->texec = nullptr;
      return fail(NKB_ERR_CUDA, std::string("timing graph instantiate: ") + cudaGetErrorString(e));
    }
    plan->tkey = base;
  }
  NKB_CUDA_TRY(cudaGraphLaunch(plan->texec, st));
  NKB_CUDA_TRY(cudaStreamSynchronize(st));
  NKB_CUDA_TRY(cudaEventElapsedTime(total_ms, plan->tev[0], plan->tev[n]));
  for (size_t i = 0; i < n; ++i) NKB_CUDA_TRY(cudaEventElapsedTime(&step_ms[i], plan->tev[i], plan->tev[i + 1]));
  return NKB_OK;
}

namespace {
// Reads every 16 bytes of a buffer (the result is never stored: the
// comparison is false for the values written before it).
__global__ void l2_read_kernel(const uint4 *p, size_t n, uint4 *sink) {
  uint32_t acc = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = p[i];
    acc |= v.x | v.y | v.z | v.w;
  }
  if (acc == 0xffffffffu) *sink = make_uint4(acc, 0, 0, 0);
}

// Evicts the plan's data from L2: writes a buffer larger than L2, then reads it
// back, so the lines left behind are clean and no write-back of the flush
// lands inside the timed launches.
void flush_l2(void *scratch, size_t bytes, cudaStream_t st) {
  cudaMemsetAsync(scratch, 0, bytes, st);
  l2_read_kernel<<<nkb::num_sms(g_rt.device) * 8, 256, 0, st>>>(static_cast<const uint4 *>(scratch), bytes / 16 - 1,
                                                               static_cast<uint4 *>(scratch) + bytes / 16 - 1);
}
}  // namespace

extern "C" int nkb_trace_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                                 float *start_ms, float *dur_ms) {
  if (int s = ensure_init()) return s;
  if (!plan || !start_ms || !dur_ms) return fail(NKB_ERR_INVALID, "bad trace arguments");
  std::vector<void *> base;
  if (int s = resolve_io(plan, ins, n_in, outs, n_out, base)) return s;
  const size_t n = plan->steps.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto &e : ev) NKB_CUDA_TRY(cudaEventCreate(&e));
  std::vector<void *> ptrs;
  int status = NKB_OK;
  cudaEventRecord(ev[0], g_rt.stream);
  for (size_t i = 0; i < n && !status; ++i) {
    const nkb::Step &st = plan->steps[i];
    ptrs.resize(st.buf_ids.size());
    for (size_t j = 0; j < st.buf_ids.size(); ++j)
      ptrs[j] = static_cast<char *>(base[st.buf_ids[j]]) + st.buf_offsets[j];
    nkb::LaunchArgs a{&st, ptrs.data(), g_rt.stream, plan->comm ? (void *)plan->comm : nullptr, plan->device};
    nvtxRangePushA(st.kernel.c_str());
    status = plan->entries[i]->launch(a);
    nvtxRangePop();
    cudaEventRecord(ev[i + 1], g_rt.stream);
  }
  cudaError_t e = cudaStreamSynchronize(g_rt.stream);
  if (!status && e != cudaSuccess) status = fail(NKB_ERR_CUDA, std::string("traced execute: ") + cudaGetErrorString(e));
  for (size_t i = 0; i < n && !status; ++i) {
    cudaEventElapsedTime(&start_ms[i], ev[0], ev[i]);
    cudaEventElapsedTime(&dur_ms[i], ev[i], ev[i + 1]);
  }
  for (auto &x : ev) cudaEventDestroy(x);
  return status;
}

extern "C" int nkb_time_steps(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out, int iters,
                              float *step_ms) {
  if (int s = ensure_init()) return s;
  if (!plan || iters < 1 || !step_ms) return fail(NKB_ERR_INVALID, "bad timing arguments");
  std::vector<void *> base;
  if (int s = resolve_io(plan, ins, n_in, outs, n_out, base)) return s;
  const size_t n = plan->steps.size();
  constexpr size_t kFlushBytes = size_t(256) << 20;
  void *scratch = nullptr;
  NKB_CUDA_TRY(cudaMalloc(&scratch, kFlushBytes));
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto &e : ev) NKB_CUDA_TRY(cudaEventCreate(&e));
  std::vector<double> acc(n, 0.0);
  std::vector<void *> ptrs;
  int status = NKB_OK;
  for (int it = 0; it < iters && !status; ++it) {
    // the flush also keeps the stream busy while the launches below are queued,
    // so no host launch latency falls between the events
    flush_l2(scratch, kFlushBytes, g_rt.stream);
    cudaEventRecord(ev[0], g_rt.stream);
    for (size_t i = 0; i < n && !status; ++i) {
      const nkb::Step &st = plan->steps[i];
      ptrs.resize(st.buf_ids.size());
      for (size_t j = 0; j < st.buf_ids.size(); ++j)
        ptrs[j] = static_cast<char *>(base[st.buf_ids[j]]) + st.buf_offsets[j];
      nkb::LaunchArgs a{&st, ptrs.data(), g_rt.stream, plan->comm ? (void *)plan->comm : nullptr, plan->device};
      status = plan->entries[i]->launch(a);
      cudaEventRecord(ev[i + 1], g_rt.stream);
    }
    cudaError_t e = cudaStreamSynchronize(g_rt.stream);
    if (!status && e != cudaSuccess) status = fail(NKB_ERR_CUDA, std::string("timed steps: ") + cudaGetErrorString(e));
    for (size_t i = 0; i < n && !status; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
      acc[i] += ms;
    }
  }
  for (auto &x : ev) cudaEventDestroy(x);
  cudaFree(scratch);
  if (!status)
    for (size_t i = 0; i < n; ++i) step_ms[i] = (float)(acc[i] / iters);
  return status;
}
