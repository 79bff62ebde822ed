// Chain compiler for the fused elementwise kernels: turns one "ew" step (its
// register program, shapes, strides and offsets) into CUDA C++ source for a
// kernel specialised to that step, compiles it for sm_100a with NVRTC at plan
// load and launches it in place of the interpreter (k_elementwise.cu).
//
// The interpreter pays, per run of VEC elements, the index decomposition with
// run-time divisors, an operand fetch and an opcode dispatch per instruction;
// on a short chain that makes it issue-bound (about 150 thread instructions per
// element for silu(gate) * up).  The specialised kernel has the shapes and
// strides as constants (divisions by constants, folded zero strides), the
// program as straight-line code on registers and the loads and stores fixed to
// their dtypes, so what is left is the arithmetic and the 16-byte memory ops.
//
// Same semantics as the interpreter's row-run kernel, instruction for
// instruction: values are 32-bit registers (fp32 for float dtypes, int32 for
// integers and bools), bf16/fp16-typed results are rounded after each node, and
// the source is compiled without contraction (--fmad=false), so each multiply
// and add rounds on its own as NumPy's per-op evaluation does.
//
// NVRTC is opened with dlopen; where it is missing, compilation fails, or the
// step's module is not loaded in the current context while a graph is being
// captured, the step runs on the interpreter kernel.  NKB_EW_JIT=0 turns the
// compiler off.

#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ew_program.cuh"

namespace nkb {
namespace ew {
namespace {

// Device code shared by every generated kernel: loads and stores of VEC
// consecutive elements of one dtype (16-byte vectors when the address allows),
// the rounding helpers and one function per opcode (opN = opcode N, the same
// expressions as the interpreter's `compute`).
const char *kPrelude = R"(
typedef unsigned int u32;
typedef unsigned long long u64;
struct EwPtrs { void *out; const void *in[8]; };
__device__ __forceinline__ float F(u32 x) { return __uint_as_float(x); }
__device__ __forceinline__ u32 U(float x) { return __float_as_uint(x); }
__device__ __forceinline__ int I(u32 x) { return (int)x; }
__device__ __forceinline__ float bf2f(unsigned short h) { return __uint_as_float(((u32)h) << 16); }
__device__ __forceinline__ unsigned short f2bf(float x) { unsigned short h; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(x)); return h; }
__device__ __forceinline__ float h2f(unsigned short h) { float r; asm("cvt.f32.f16 %0, %1;" : "=f"(r) : "h"(h)); return r; }
__device__ __forceinline__ unsigned short f2h(float x) { unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(x)); return h; }
__device__ __forceinline__ u32 rbf(u32 x) { return U(bf2f(f2bf(F(x)))); }
__device__ __forceinline__ u32 rhf(u32 x) { return U(h2f(f2h(F(x)))); }
#define QNAN __int_as_float(0x7fc00000)
#define IMIN (-2147483647 - 1)

template <int DT> __device__ __forceinline__ u32 ld1(const void *p, long long i) {
  if (DT == 0) return ((const u32 *)p)[i];
  if (DT == 1) return U(bf2f(((const unsigned short *)p)[i]));
  if (DT == 2) return U(h2f(((const unsigned short *)p)[i]));
  if (DT == 3 || DT == 4) return ((const u32 *)p)[i];
  if (DT == 5) return (u32)(int)((const signed char *)p)[i];
  if (DT == 6) return ((const unsigned char *)p)[i];
  if (DT == 7) return ((const unsigned char *)p)[i] ? 1u : 0u;
  if (DT == 8) return (u32)(int)((const short *)p)[i];
  if (DT == 9) return ((const unsigned short *)p)[i];
  return 0u;
}
template <int DT> __device__ __forceinline__ void st1(void *p, long long i, u32 v) {
  if (DT == 0 || DT == 3 || DT == 4) ((u32 *)p)[i] = v;
  else if (DT == 1) ((unsigned short *)p)[i] = f2bf(F(v));
  else if (DT == 2) ((unsigned short *)p)[i] = f2h(F(v));
  else if (DT == 5 || DT == 6) ((unsigned char *)p)[i] = (unsigned char)v;
  else if (DT == 7) ((unsigned char *)p)[i] = v ? 1 : 0;
  else if (DT == 8 || DT == 9) ((unsigned short *)p)[i] = (unsigned short)v;
}
template <int DT, long long ST, class IDX> __device__ __forceinline__ void ld(const void *p, IDX off, u32 (&d)[VEC]) {
  if (ST == 0) {
    const u32 x = ld1<DT>(p, off);
#pragma unroll
    for (int v = 0; v < VEC; ++v) d[v] = x;
    return;
  }
  if (ST == 1 && (DT == 0 || DT == 3 || DT == 4) && (((u64)((const u32 *)p + off)) & 15) == 0) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      const uint4 t = *(const uint4 *)((const u32 *)p + off + k);
      d[k] = t.x; d[k + 1] = t.y; d[k + 2] = t.z; d[k + 3] = t.w;
    }
    return;
  }
  if (ST == 1 && DT == 1 && (((u64)((const unsigned short *)p + off)) & (2 * VEC - 1)) == 0) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      const uint2 t = *(const uint2 *)((const unsigned short *)p + off + k);
      d[k] = t.x << 16; d[k + 1] = t.x & 0xffff0000u; d[k + 2] = t.y << 16; d[k + 3] = t.y & 0xffff0000u;
    }
    return;
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) d[v] = ld1<DT>(p, off + (IDX)v * (IDX)ST);
}
template <int DT, long long ST, class IDX> __device__ __forceinline__ void st(void *p, IDX off, const u32 (&x)[VEC]) {
  if (ST == 1 && (DT == 0 || DT == 3 || DT == 4) && (((u64)((u32 *)p + off)) & 15) == 0) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      uint4 t;
      t.x = x[k]; t.y = x[k + 1]; t.z = x[k + 2]; t.w = x[k + 3];
      *(uint4 *)((u32 *)p + off + k) = t;
    }
    return;
  }
  if (ST == 1 && DT == 1 && (((u64)((unsigned short *)p + off)) & 7) == 0) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      uint2 t;
      t.x = (u32)f2bf(F(x[k])) | ((u32)f2bf(F(x[k + 1])) << 16);
      t.y = (u32)f2bf(F(x[k + 2])) | ((u32)f2bf(F(x[k + 3])) << 16);
      *(uint2 *)((unsigned short *)p + off + k) = t;
    }
    return;
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) st1<DT>(p, off + (IDX)v * (IDX)ST, x[v]);
}

#define OP(n, e) __device__ __forceinline__ u32 op##n(u32 a, u32 b, u32 c) { return (e); }
OP(10, U(F(a) + F(b)))
OP(11, U(F(a) - F(b)))
OP(12, U(F(a) * F(b)))
OP(13, U(F(a) / F(b)))
OP(14, U(powf(F(a), F(b))))
OP(15, U((F(a) != F(a) || F(b) != F(b)) ? QNAN : fmaxf(F(a), F(b))))
OP(16, U((F(a) != F(a) || F(b) != F(b)) ? QNAN : fminf(F(a), F(b))))
OP(17, U(atan2f(F(a), F(b))))
OP(18, U(fmodf(F(a), F(b))))
OP(20, U(-F(a)))
OP(21, U(fabsf(F(a))))
OP(22, U(__expf(F(a))))
OP(23, U(logf(F(a))))
OP(24, U(sqrtf(F(a))))
OP(25, U(1.0f / sqrtf(F(a))))
OP(26, U(tanhf(F(a))))
OP(27, U(sinf(F(a))))
OP(28, U(cosf(F(a))))
OP(29, U(floorf(F(a))))
OP(30, U(ceilf(F(a))))
OP(31, U(F(a) > 0.f ? 1.f : (F(a) < 0.f ? -1.f : F(a))))
OP(32, rbf(a))
OP(33, rhf(a))
OP(34, U(__frcp_rn(F(a))))
OP(40, (u32)(F(a) == F(b)))
OP(41, (u32)(F(a) != F(b)))
OP(42, (u32)(F(a) < F(b)))
OP(43, (u32)(F(a) <= F(b)))
OP(44, (u32)(F(a) > F(b)))
OP(45, (u32)(F(a) >= F(b)))
OP(50, a + b)
OP(51, a - b)
OP(52, a * b)
OP(53, (u32)(I(b) == 0 ? -1 : (I(a) == IMIN && I(b) == -1 ? I(a) : I(a) / I(b))))
OP(54, (u32)max(I(a), I(b)))
OP(55, (u32)min(I(a), I(b)))
OP(56, a & b)
OP(57, a | b)
OP(58, a ^ b)
OP(59, (u32)(I(b) == 0 ? I(a) : (I(b) == -1 ? 0 : I(a) % I(b))))
OP(60, (u32)(-I(a)))
OP(61, (u32)(I(a) < 0 ? -I(a) : I(a)))
OP(62, ~a)
OP(63, (u32)(I(a) > 0 ? 1 : (I(a) < 0 ? -1 : 0)))
OP(64, b < 32 ? a << b : 0u)
OP(65, b < 32 ? (u32)(I(a) >> b) : (I(a) < 0 ? 0xffffffffu : 0u))
OP(70, (u32)(a == b))
OP(71, (u32)(a != b))
OP(72, (u32)(I(a) < I(b)))
OP(73, (u32)(I(a) <= I(b)))
OP(74, (u32)(I(a) > I(b)))
OP(75, (u32)(I(a) >= I(b)))
OP(76, (u32)(a < b))
OP(77, (u32)(a <= b))
OP(78, (u32)(a > b))
OP(79, (u32)(a >= b))
OP(80, b == 0 ? 0xffffffffu : a / b)
OP(81, max(a, b))
OP(82, min(a, b))
OP(83, b == 0 ? a : a % b)
OP(90, a ? b : c)
OP(100, (u32)(F(a) != F(a) ? 0 : (F(a) >= 2147483648.f ? 2147483647 : (F(a) <= -2147483648.f ? IMIN : (int)F(a)))))
OP(101, U((float)I(a)))
OP(102, U((float)a))
OP(103, (F(a) != F(a) || F(a) <= 0.f) ? 0u : (F(a) >= 4294967296.f ? 0xffffffffu : (u32)F(a)))
OP(104, (u32)(a != 0u))
OP(105, (u32)(F(a) != 0.f))
)";

bool known_op(int op) {
  return (op >= FADD && op <= FREM) || (op >= FNEG && op <= FRCP) || (op >= FEQ && op <= FGE) ||
         (op >= IADD && op <= IREM) || (op >= INEG && op <= ISIGN) || op == ISHL || op == ISHR ||
         (op >= IEQ && op <= UREM) || op == SEL || (op >= F2I && op <= FNZ) || op == CF || op == CI ||
         op == LD || op == IOTA;
}

struct Kernel {
  std::string key;                      // the generated kernel body (without the prelude)
  std::vector<char> cubin;              // empty when compilation failed
  struct Loaded {
    unsigned long long ctx_id;  // cuCtxGetId: unique for the process's life (a handle may be reused)
    CUfunction fn;
    int per_sm;  // resident CTAs of 256 threads per SM
  };
  std::vector<Loaded> loaded;
  int vec = 8;
  int64_t runs = 0;
};

struct Nvrtc {
  bool tried = false, ok = false;
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
};

// Driver calls, resolved through the runtime so the library does not link
// libcuda directly (it loads on hosts without a driver).
struct Driver {
  bool ok = false;
  decltype(&cuCtxGetCurrent) ctx_current = nullptr;
  decltype(&cuCtxGetId) ctx_id = nullptr;
  decltype(&cuModuleLoadData) module_load = nullptr;
  decltype(&cuModuleGetFunction) module_function = nullptr;
  decltype(&cuLaunchKernel) launch = nullptr;
  decltype(&cuGetErrorString) error_string = nullptr;
  decltype(&cuOccupancyMaxActiveBlocksPerMultiprocessor) occupancy = nullptr;
};

const Driver &driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char *name) -> void * {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
      }
      return p;
    };
    d.ctx_current = reinterpret_cast<decltype(d.ctx_current)>(get("cuCtxGetCurrent"));
    d.ctx_id = reinterpret_cast<decltype(d.ctx_id)>(get("cuCtxGetId"));
    d.module_load = reinterpret_cast<decltype(d.module_load)>(get("cuModuleLoadData"));
    d.module_function = reinterpret_cast<decltype(d.module_function)>(get("cuModuleGetFunction"));
    d.launch = reinterpret_cast<decltype(d.launch)>(get("cuLaunchKernel"));
    d.error_string = reinterpret_cast<decltype(d.error_string)>(get("cuGetErrorString"));
    d.occupancy = reinterpret_cast<decltype(d.occupancy)>(get("cuOccupancyMaxActiveBlocksPerMultiprocessor"));
    d.ok = d.ctx_current && d.ctx_id && d.module_load && d.module_function && d.launch && d.error_string && d.occupancy;
  });
  return d;
}

std::mutex g_mu;
Nvrtc g_rtc;
std::map<std::string, Kernel *> g_by_source;                // generated kernel body -> kernel
std::map<std::vector<int64_t>, Kernel *> g_by_step;          // step parameters -> kernel (null: not taken)
int64_t g_compiled = 0, g_failed = 0, g_launched = 0;

bool enabled() {
  static const bool on = [] {
    const char *e = getenv("NKB_EW_JIT");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool open_nvrtc() {
  if (g_rtc.tried) return g_rtc.ok;
  g_rtc.tried = true;
  void *h = nullptr;
  for (const char *n : {"libnvrtc.so.12", "libnvrtc.so"})
    if ((h = dlopen(n, RTLD_NOW | RTLD_LOCAL))) break;
  if (!h) return false;
#define SYM(f, n) g_rtc.f = reinterpret_cast<decltype(g_rtc.f)>(dlsym(h, n))
  SYM(create, "nvrtcCreateProgram");
  SYM(compile, "nvrtcCompileProgram");
  SYM(log_size, "nvrtcGetProgramLogSize");
  SYM(log, "nvrtcGetProgramLog");
  SYM(cubin_size, "nvrtcGetCUBINSize");
  SYM(cubin, "nvrtcGetCUBIN");
  SYM(destroy, "nvrtcDestroyProgram");
#undef SYM
  g_rtc.ok = g_rtc.create && g_rtc.compile && g_rtc.log_size && g_rtc.log && g_rtc.cubin_size && g_rtc.cubin &&
             g_rtc.destroy;
  return g_rtc.ok;
}

// Registers the program reads or writes (the interpreter's register-file size).
int program_regs(const Params &p) {
  int n = p.out_reg + 1;
  for (int i = 0; i < p.n_instr; ++i) {
    const Instr &I = p.prog[i];
    n = max(n, (int)I.dst + 1);
    if (I.op != LD && I.op != IOTA && I.op != CF && I.op != CI) {
      n = max(n, (int)I.a + 1);
      if (!I.bimm) n = max(n, (int)I.b + 1);
      if (I.op == SEL) n = max(n, (int)I.c + 1);
    }
  }
  return n;
}

std::string lit(int64_t v) { return "(IDX)" + std::to_string(v) + "LL"; }

// CUDA C++ source of the kernel for one step, or "" when the step is not one
// the compiler takes (the interpreter keeps it).
std::string generate(const Params &p, int *vec_out) {
  const int last = p.rank - 1;
  const int64_t inner = p.shape[last];
  if (p.n <= 0 || inner % 4 != 0) return "";
  for (int i = 0; i < p.n_instr; ++i)
    if (!known_op(p.prog[i].op)) return "";
  for (int k = 0; k < p.n_in; ++k)
    if (p.in_dtype[k] < 0 || p.in_dtype[k] > 9) return "";
  if (p.out_dtype < 0 || p.out_dtype > 9) return "";
  const int vec = inner % 8 == 0 ? 8 : 4;
  *vec_out = vec;
  // 32-bit index math when every offset the kernel forms fits
  auto span_of = [&](int64_t off, const int64_t *st) {
    int64_t s = off < 0 ? -off : off;
    for (int d = 0; d < p.rank; ++d) s += (p.shape[d] - 1) * (st[d] < 0 ? -st[d] : st[d]);
    return s;
  };
  int64_t span = p.n + vec;
  span = max(span, span_of(p.out_off, p.out_strides) + vec);
  for (int k = 0; k < p.n_in; ++k) span = max(span, span_of(p.in_off[k], p.in_strides[k]) + vec);
  const bool small = span < (int64_t)INT32_MAX / 2;
  bool iota = false;
  for (int i = 0; i < p.n_instr; ++i) iota |= p.prog[i].op == IOTA;

  std::string s;
  s.reserve(4096);
  s += "// VEC " + std::to_string(vec) + "\n";  // the body alone is the cache key; the prelude is added to compile
  s += "extern \"C\" __global__ void __launch_bounds__(256) ew_gen(const EwPtrs p) {\n";
  s += std::string("  typedef ") + (small ? "int" : "long long") + " IDX;\n";
  const int64_t rpr = inner / vec, runs = p.n / vec;
  s += "  for (IDX c = (IDX)blockIdx.x * 256 + threadIdx.x; c < " + lit(runs) + "; c += (IDX)gridDim.x * 256) {\n";
  if (last == 0) {
    s += "    const IDX col = c * VEC;\n";
  } else {
    s += "    const IDX row = c / " + lit(rpr) + ";\n";
    s += "    const IDX col = (c - row * " + lit(rpr) + ") * VEC;\n";
  }
  auto base_expr = [&](int64_t off, int64_t st_last) {
    std::string e = lit(off);
    if (st_last) e += " + col * " + lit(st_last);
    return e;
  };
  s += "    IDX o = " + base_expr(p.out_off, p.out_strides[last]) + ";\n";
  for (int k = 0; k < p.n_in; ++k)
    s += "    IDX b" + std::to_string(k) + " = " + base_expr(p.in_off[k], p.in_strides[k][last]) + ";\n";
  if (last > 0) {
    s += "    IDX rem = row;\n";
    for (int d = last - 1; d >= 0; --d) {
      const std::string id = "i" + std::to_string(d);
      if (d == 0) {
        s += "    const IDX " + id + " = rem;\n";
      } else {
        s += "    const IDX " + id + " = rem % " + lit(p.shape[d]) + ";\n";
        s += "    rem = rem / " + lit(p.shape[d]) + ";\n";
      }
      if (p.out_strides[d]) s += "    o += " + id + " * " + lit(p.out_strides[d]) + ";\n";
      for (int k = 0; k < p.n_in; ++k)
        if (p.in_strides[k][d]) s += "    b" + std::to_string(k) + " += " + id + " * " + lit(p.in_strides[k][d]) + ";\n";
      if (!iota) s += "    (void)" + id + ";\n";
    }
  }
  const int nregs = program_regs(p);
  for (int g = 0; g < nregs; ++g) s += "    u32 r" + std::to_string(g) + "[VEC] = {};\n";
  auto R = [](int g) { return "r" + std::to_string(g); };
  for (int i = 0; i < p.n_instr; ++i) {
    const Instr &I = p.prog[i];
    if (I.op == LD) {
      s += "    ld<" + std::to_string(p.in_dtype[I.a]) + ", " + std::to_string(p.in_strides[I.a][last]) + "LL>(p.in[" +
           std::to_string(I.a) + "], b" + std::to_string(I.a) + ", " + R(I.dst) + ");\n";
      continue;
    }
    s += "#pragma unroll\n    for (int v = 0; v < VEC; ++v) {\n";
    if (I.op == IOTA) {
      if (I.a == last)
        s += "      " + R(I.dst) + "[v] = (u32)(int)(col + v);\n";
      else
        s += "      " + R(I.dst) + "[v] = (u32)(int)i" + std::to_string(I.a) + ";\n";
      s += "    }\n";
      continue;
    }
    char imm[24];
    snprintf(imm, sizeof imm, "0x%08xu", I.imm);
    if (I.op == CF || I.op == CI) {
      s += "      " + R(I.dst) + "[v] = " + imm + ";\n";
    } else {
      const std::string a = R(I.a) + "[v]";
      const std::string b = I.bimm ? std::string(imm) : R(I.b) + "[v]";
      const std::string c = I.op == SEL ? R(I.c) + "[v]" : std::string("0u");
      s += "      " + R(I.dst) + "[v] = op" + std::to_string(I.op) + "(" + a + ", " + b + ", " + c + ");\n";
    }
    if (I.rnd == 1) s += "      " + R(I.dst) + "[v] = rbf(" + R(I.dst) + "[v]);\n";
    if (I.rnd == 2) s += "      " + R(I.dst) + "[v] = rhf(" + R(I.dst) + "[v]);\n";
    s += "    }\n";
  }
  s += "    st<" + std::to_string(p.out_dtype) + ", " + std::to_string(p.out_strides[last]) + "LL>(p.out, o, " +
       R(p.out_reg) + ");\n";
  s += "  }\n}\n";
  return s;
}

bool compile(Kernel *k) {
  if (!open_nvrtc()) return false;
  nvrtcProgram prog = nullptr;
  const std::string src = "#define VEC " + std::to_string(k->vec) + "\n" + kPrelude + k->key;
  if (g_rtc.create(&prog, src.c_str(), "ew_gen.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) return false;
  const char *opts[] = {"--gpu-architecture=sm_100a", "--fmad=false", "-default-device", "--std=c++17"};
  const nvrtcResult r = g_rtc.compile(prog, 4, opts);
  bool ok = r == NVRTC_SUCCESS;
  if (!ok) {
    size_t n = 0;
    g_rtc.log_size(prog, &n);
    std::string log(n, '\0');
    if (n) g_rtc.log(prog, &log[0]);
    if (getenv("NKB_EW_JIT_LOG")) fprintf(stderr, "nkb ew compiler:\n%s\n%s\n", src.c_str(), log.c_str());
  } else {
    size_t n = 0;
    ok = g_rtc.cubin_size(prog, &n) == NVRTC_SUCCESS && n > 0;
    if (ok) {
      k->cubin.resize(n);
      ok = g_rtc.cubin(prog, k->cubin.data()) == NVRTC_SUCCESS;
    }
  }
  g_rtc.destroy(&prog);
  if (!ok) k->cubin.clear();
  return ok;
}

// The kernel's function in the current context, loading the module when
// `may_load` (never while a graph is being captured).
const Kernel::Loaded *function_in_context(Kernel *k, bool may_load) {
  const Driver &drv = driver();
  if (k->cubin.empty() || !drv.ok) return nullptr;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (drv.ctx_current(&ctx) != CUDA_SUCCESS || !ctx || drv.ctx_id(ctx, &id) != CUDA_SUCCESS) return nullptr;
  for (auto &e : k->loaded)
    if (e.ctx_id == id) return &e;
  if (!may_load) return nullptr;
  CUmodule mod = nullptr;
  CUfunction fn = nullptr;
  if (drv.module_load(&mod, k->cubin.data()) != CUDA_SUCCESS) return nullptr;
  if (drv.module_function(&fn, mod, "ew_gen") != CUDA_SUCCESS) return nullptr;
  int per_sm = 0;
  if (drv.occupancy(&per_sm, fn, 256, 0) != CUDA_SUCCESS || per_sm < 1) per_sm = 1;
  k->loaded.push_back(Kernel::Loaded{id, fn, per_sm});
  return &k->loaded.back();
}

// The kernel for a step (its parameters `ints`, parsed into `p`), generated
// and compiled on first sight; null when the compiler does not take the step.
Kernel *kernel_for(const Params &p, const std::vector<int64_t> &ints) {
  auto hit = g_by_step.find(ints);
  if (hit != g_by_step.end()) return hit->second;
  int vec = 8;
  std::string body = generate(p, &vec);
  Kernel *k = nullptr;
  if (!body.empty()) {
    auto it = g_by_source.find(body);
    if (it != g_by_source.end()) {
      k = it->second;
    } else {
      k = new Kernel;  // kept for the life of the process (modules stay loaded)
      k->key = std::move(body);
      k->vec = vec;
      k->runs = p.n / vec;
      if (compile(k)) ++g_compiled;
      else ++g_failed;
      g_by_source.emplace(k->key, k);
    }
  }
  g_by_step.emplace(ints, k);
  return k;
}

}  // namespace

int jit_prepare(const Params &p, const std::vector<int64_t> &ints) {
  if (!enabled()) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  Kernel *k = kernel_for(p, ints);
  if (!k) return 0;
  return function_in_context(k, true) ? 1 : 0;
}

int jit_compiled(const Params &p, const std::vector<int64_t> &ints) {
  if (!enabled()) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  Kernel *k = kernel_for(p, ints);
  return k && !k->cubin.empty() ? 1 : 0;
}

int jit_launch(const Params &p, const std::vector<int64_t> &ints, cudaStream_t stream, int device, bool *launched) {
  *launched = false;
  if (!enabled()) return NKB_OK;
  Kernel::Loaded fn{};  // copied under the lock (the vector may grow later)
  Kernel *k = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    k = kernel_for(p, ints);
    if (!k) return NKB_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
      cudaGetLastError();
      return NKB_OK;
    }
    const Kernel::Loaded *l = function_in_context(k, cs == cudaStreamCaptureStatusNone);
    if (!l) return NKB_OK;
    fn = *l;
    ++g_launched;
  }
  struct {
    void *out;
    const void *in[kMaxIn];
  } ptrs;
  ptrs.out = p.out;
  for (int i = 0; i < kMaxIn; ++i) ptrs.in[i] = i < p.n_in ? p.in[i] : nullptr;
  void *args[] = {&ptrs};
  int64_t blocks = (k->runs + 255) / 256;
  // one wave of resident CTAs, each striding over the runs
  const int64_t cap = (int64_t)num_sms(device) * fn.per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const Driver &drv = driver();
  const CUresult r = drv.launch(fn.fn, (unsigned)blocks, 1, 1, 256, 1, 1, 0, (CUstream)stream, args, nullptr);
  if (r != CUDA_SUCCESS) {
    const char *m = nullptr;
    drv.error_string(r, &m);
    return fail(NKB_ERR_CUDA, std::string("ew_gen launch: ") + (m ? m : "unknown error"));
  }
  *launched = true;
  return NKB_OK;
}

}  // namespace ew
}  // namespace nkb

// Counters of the chain compiler since the library was loaded: programs
// compiled, programs the compiler could not take (left to the interpreter) and
// launches of compiled kernels (issued, or captured into a graph; replays of a
// captured graph are not counted).
extern "C" NKB_API int nkb_ew_compiler_stats(int64_t *compiled, int64_t *failed, int64_t *launched) {
  std::lock_guard<std::mutex> lk(nkb::ew::g_mu);
  if (compiled) *compiled = nkb::ew::g_compiled;
  if (failed) *failed = nkb::ew::g_failed;
  if (launched) *launched = nkb::ew::g_launched;
  return NKB_OK;
}
