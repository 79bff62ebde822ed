// Fused elementwise chains: one launch evaluates a whole group of traced
// elementwise nodes (add/multiply/exponential/compare/select/convert ...,
// core/ops/binary.py + unary.py + indexing.py:20-110 of the reference) over
// the output's index space.
//
// Every operand is a strided view of a device buffer (offset + per-axis
// element strides), so broadcast (stride 0), transpose, slice and reshape of
// a dense buffer cost no copy: they are folded into the view by the planner.
// The group's arithmetic is a short register program.  Where the innermost
// axis has a multiple of 4 elements the step normally runs on a kernel
// compiled for it at plan load (ew_jit.cu); this file is the interpreter that
// decodes the program from the kernel parameters at run time, used for the
// other steps and wherever the compiler does not take one.  Registers hold
// 32-bit values: fp32 for every float dtype, int32 for integers and bools.
// Results of bf16/fp16-typed nodes are rounded to that type after each node
// (program op RBF/RF16), matching NumPy's per-op rounding.
//
// Hot path: when every operand is either dense over the output or a scalar,
// the offsets are affine in the flat index and each thread works on VEC
// consecutive elements with no index decomposition.

#include <math.h>

#include "common.cuh"
#include "ew_program.cuh"

namespace nkb {
namespace ew {

__device__ __forceinline__ float rnd_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float rnd_f16(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float fsignf(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : x); }

// One arithmetic instruction on VEC lanes held in (real) registers.  Loads
// and iota are executed by the callers, which know the addressing.
template <int VEC>
__device__ __forceinline__ void compute(const Instr I, const uint32_t (&A)[VEC], const uint32_t (&B)[VEC],
                                        const uint32_t (&C)[VEC], uint32_t (&d)[VEC]) {
  {
#define LANES _Pragma("unroll") for (int v = 0; v < VEC; ++v)
#define FA __uint_as_float(A[v])
#define FB __uint_as_float(B[v])
#define IA static_cast<int32_t>(A[v])
#define IB static_cast<int32_t>(B[v])
#define SETF(x) d[v] = __float_as_uint(x)
#define SETI(x) d[v] = static_cast<uint32_t>(x)
    switch (I.op) {
      case CF: case CI: LANES d[v] = I.imm; break;
      case FADD: LANES SETF(FA + FB); break;
      case FSUB: LANES SETF(FA - FB); break;
      case FMUL: LANES SETF(FA * FB); break;
      case FDIV: LANES SETF(FA / FB); break;
      case FPOW: LANES SETF(powf(FA, FB)); break;
      case FMAX: LANES SETF((FA != FA || FB != FB) ? __int_as_float(0x7fc00000) : fmaxf(FA, FB)); break;
      case FMIN: LANES SETF((FA != FA || FB != FB) ? __int_as_float(0x7fc00000) : fminf(FA, FB)); break;
      case FATAN2: LANES SETF(atan2f(FA, FB)); break;
      case FREM: LANES SETF(fmodf(FA, FB)); break;
      case FNEG: LANES SETF(-FA); break;
      case FABS: LANES SETF(fabsf(FA)); break;
      // exp as ex2.approx of the scaled argument: relative error about |x| * 6e-8 + 2e-7
      // (below the 1e-5 bar of fp32 elementwise work for every non-overflowing x)
      case FEXP: LANES SETF(__expf(FA)); break;
      case FLOG: LANES SETF(logf(FA)); break;
      case FSQRT: LANES SETF(sqrtf(FA)); break;
      case FRSQRT: LANES SETF(1.0f / sqrtf(FA)); break;
      case FTANH: LANES SETF(tanhf(FA)); break;
      case FSIN: LANES SETF(sinf(FA)); break;
      case FCOS: LANES SETF(cosf(FA)); break;
      case FFLOOR: LANES SETF(floorf(FA)); break;
      case FCEIL: LANES SETF(ceilf(FA)); break;
      case FSIGN: LANES SETF(fsignf(FA)); break;
      case RBF: LANES SETF(rnd_bf16(FA)); break;
      case RF16: LANES SETF(rnd_f16(FA)); break;
      case FRCP: LANES SETF(__frcp_rn(FA)); break;  // correctly rounded, as 1.0f / x
      case FEQ: LANES SETI(FA == FB); break;
      case FNE: LANES SETI(FA != FB); break;
      case FLT: LANES SETI(FA < FB); break;
      case FLE: LANES SETI(FA <= FB); break;
      case FGT: LANES SETI(FA > FB); break;
      case FGE: LANES SETI(FA >= FB); break;
      case IADD: LANES SETI(A[v] + B[v]); break;
      case ISUB: LANES SETI(A[v] - B[v]); break;
      case IMUL: LANES SETI(A[v] * B[v]); break;
      case IDIV: LANES SETI(IB == 0 ? -1 : (IA == INT32_MIN && IB == -1 ? IA : IA / IB)); break;
      case IREM: LANES SETI(IB == 0 ? IA : (IB == -1 ? 0 : IA % IB)); break;
      case IMAX: LANES SETI(max(IA, IB)); break;
      case IMIN: LANES SETI(min(IA, IB)); break;
      case IAND: LANES SETI(A[v] & B[v]); break;
      case IOR: LANES SETI(A[v] | B[v]); break;
      case IXOR: LANES SETI(A[v] ^ B[v]); break;
      case ISHL: LANES SETI(B[v] < 32 ? A[v] << B[v] : 0u); break;
      case ISHR: LANES SETI(B[v] < 32 ? (uint32_t)(IA >> B[v]) : (IA < 0 ? 0xffffffffu : 0u)); break;
      case INEG: LANES SETI(-IA); break;
      case IABS: LANES SETI(IA < 0 ? -IA : IA); break;
      case INOT: LANES SETI(~A[v]); break;
      case ISIGN: LANES SETI(IA > 0 ? 1 : (IA < 0 ? -1 : 0)); break;
      case IEQ: LANES SETI(A[v] == B[v]); break;
      case INE: LANES SETI(A[v] != B[v]); break;
      case ILT: LANES SETI(IA < IB); break;
      case ILE: LANES SETI(IA <= IB); break;
      case IGT: LANES SETI(IA > IB); break;
      case IGE: LANES SETI(IA >= IB); break;
      case ULT: LANES SETI(A[v] < B[v]); break;
      case ULE: LANES SETI(A[v] <= B[v]); break;
      case UGT: LANES SETI(A[v] > B[v]); break;
      case UGE: LANES SETI(A[v] >= B[v]); break;
      case UDIV: LANES SETI(B[v] == 0 ? 0xffffffffu : A[v] / B[v]); break;
      case UREM: LANES SETI(B[v] == 0 ? A[v] : A[v] % B[v]); break;
      case UMAX: LANES SETI(max(A[v], B[v])); break;
      case UMIN: LANES SETI(min(A[v], B[v])); break;
      case SEL: LANES d[v] = A[v] ? B[v] : C[v]; break;
      case F2I: {
        // float -> int32, truncating; NaN -> 0, saturating at the int32 range
        LANES {
          float f = FA;
          int32_t x = (f != f) ? 0 : (f >= 2147483648.f ? INT32_MAX : (f <= -2147483648.f ? INT32_MIN : (int32_t)f));
          SETI(x);
        }
        break;
      }
      case F2U: {
        LANES {
          float f = FA;
          uint32_t x = (f != f || f <= 0.f) ? 0u : (f >= 4294967296.f ? 0xffffffffu : (uint32_t)f);
          SETI(x);
        }
        break;
      }
      case I2F: LANES SETF((float)IA); break;
      case U2F: LANES SETF((float)A[v]); break;
      case INZ: LANES SETI(A[v] != 0u); break;
      case FNZ: LANES SETI(FA != 0.f); break;
      default: break;
    }
    if (I.rnd == 1) {
      LANES d[v] = __float_as_uint(rnd_bf16(__uint_as_float(d[v])));
    } else if (I.rnd == 2) {
      LANES d[v] = __float_as_uint(rnd_f16(__uint_as_float(d[v])));
    }
#undef LANES
#undef FA
#undef FB
#undef IA
#undef IB
#undef SETF
#undef SETI
  }
}

// Opcodes applied to the accumulator in place (operand a = the previous result).
__host__ __device__ __forceinline__ bool inplace_op(uint8_t op) {
  return op == FADD || op == FSUB || op == FMUL || op == FDIV || op == FNEG || op == FEXP || op == FRCP ||
         op == FMAX || op == FMIN;
}

template <int VEC>
__device__ __forceinline__ void compute_inplace(const Instr I, uint32_t (&x)[VEC], const uint32_t (&B)[VEC]) {
#define LANES _Pragma("unroll") for (int v = 0; v < VEC; ++v)
#define FX __uint_as_float(x[v])
#define FB __uint_as_float(B[v])
#define SETF(e) x[v] = __float_as_uint(e)
  switch (I.op) {
    case FADD: LANES SETF(FX + FB); break;
    case FSUB: LANES SETF(FX - FB); break;
    case FMUL: LANES SETF(FX * FB); break;
    case FDIV: LANES SETF(FX / FB); break;
    case FNEG: LANES SETF(-FX); break;
    case FEXP: LANES SETF(__expf(FX)); break;
    case FRCP: LANES SETF(__frcp_rn(FX)); break;
    case FMAX: LANES SETF((FX != FX || FB != FB) ? __int_as_float(0x7fc00000) : fmaxf(FX, FB)); break;
    case FMIN: LANES SETF((FX != FX || FB != FB) ? __int_as_float(0x7fc00000) : fminf(FX, FB)); break;
    default: break;
  }
  if (I.rnd == 1) {
    LANES x[v] = __float_as_uint(rnd_bf16(__uint_as_float(x[v])));
  } else if (I.rnd == 2) {
    LANES x[v] = __float_as_uint(rnd_f16(__uint_as_float(x[v])));
  }
#undef LANES
#undef FX
#undef FB
#undef SETF
}

__device__ __forceinline__ void exec_one(const Instr I, const int64_t (*idx)[kVec], uint32_t (*r)[kVec]) {
  uint32_t A[kVec], B[kVec], C[kVec], d[kVec];
#pragma unroll
  for (int v = 0; v < kVec; ++v) {
    A[v] = r[I.a][v];
    B[v] = I.bimm ? I.imm : r[I.b][v];
    C[v] = r[I.c][v];
  }
  if (I.op == IOTA) {
#pragma unroll
    for (int v = 0; v < kVec; ++v) d[v] = static_cast<uint32_t>(static_cast<int32_t>(idx[I.a][v]));
  } else {
    compute<kVec>(I, A, B, C, d);
  }
#pragma unroll
  for (int v = 0; v < kVec; ++v) r[I.dst][v] = d[v];
}

// Executes the program for VEC lanes whose per-input element offsets and
// per-axis indices are given.
__device__ __forceinline__ void run_program(const Params &p, const int64_t (*off)[kVec], const int64_t (*idx)[kVec],
                                            int nlanes, uint32_t (*r)[kVec]) {
  for (int pc = 0; pc < p.n_instr; ++pc) {
    const Instr I = p.prog[pc];
    if (I.op == LD) {
      for (int v = 0; v < kVec; ++v)
        if (v < nlanes) r[I.dst][v] = load_as_reg(p.in[I.a], off[I.a][v], p.in_dtype[I.a]);
    } else {
      exec_one(I, idx, r);
    }
  }
}

__global__ void __launch_bounds__(256) ew_kernel(const __grid_constant__ Params p) {
  uint32_t r[kRegs][kVec];
  int64_t off[kMaxIn][kVec];
  int64_t idx[kMaxRank][kVec];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * kVec;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kVec; base < p.n; base += stride) {
    const int nl = (p.n - base) < kVec ? (int)(p.n - base) : kVec;
    int64_t oo[kVec];
    if (p.contig) {
      // every operand is dense over the output or a scalar
#pragma unroll
      for (int v = 0; v < kVec; ++v) {
        const int64_t i = base + v;
        for (int k = 0; k < p.n_in; ++k) off[k][v] = p.in_off[k] + (p.in_strides[k][p.rank - 1] ? i : 0);
        oo[v] = p.out_off + i;
        for (int d = 0; d < p.rank; ++d) idx[d][v] = 0;
      }
      // axis indices are only needed by IOTA; derive them when the program uses it
      for (int pc = 0; pc < p.n_instr; ++pc)
        if (p.prog[pc].op == IOTA) {
#pragma unroll
          for (int v = 0; v < kVec; ++v) {
            int64_t rem = base + v;
            for (int d = p.rank - 1; d >= 0; --d) {
              idx[d][v] = rem % p.shape[d];
              rem /= p.shape[d];
            }
          }
          break;
        }
    } else {
#pragma unroll
      for (int v = 0; v < kVec; ++v) {
        int64_t rem = base + v;
        if (rem >= p.n) rem = p.n - 1;
        int64_t o = p.out_off;
        for (int k = 0; k < p.n_in; ++k) off[k][v] = p.in_off[k];
        for (int d = p.rank - 1; d >= 0; --d) {
          const int64_t s = p.shape[d];
          const int64_t q = rem / s;
          const int64_t id = rem - q * s;
          rem = q;
          idx[d][v] = id;
          o += id * p.out_strides[d];
          for (int k = 0; k < p.n_in; ++k) off[k][v] += id * p.in_strides[k][d];
        }
        oo[v] = o;
      }
    }
    run_program(p, off, idx, nl, r);
#pragma unroll
    for (int v = 0; v < kVec; ++v)
      if (v < nl) store_from_reg(p.out, oo[v], p.out_dtype, r[p.out_reg][v]);
  }
}

// Row-run variant: the innermost (collapsed) axis has a multiple of VEC
// elements, so each thread takes VEC consecutive elements of one row.  The
// row index is decomposed once per run (32-bit math when every offset fits);
// operands with unit inner stride are read with 16-byte vector loads,
// broadcast operands (inner stride 0) with one scalar load.  The program's
// registers live in shared memory ([reg][lane][thread], bank-conflict free),
// sized to the registers the program uses, so the interpreter state never
// spills to local memory.
template <int VEC>
__device__ __forceinline__ void load_run(const void *p, int64_t off, int64_t st, int dt, uint32_t (&d)[VEC]) {
  if (st == 0) {
    const uint32_t v = load_as_reg(p, off, dt);
#pragma unroll
    for (int k = 0; k < VEC; ++k) d[k] = v;
    return;
  }
  if (st == 1 && dt == NKB_F32 && ((reinterpret_cast<uintptr_t>(static_cast<const float *>(p) + off) & 15) == 0)) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      const uint4 t = *reinterpret_cast<const uint4 *>(static_cast<const float *>(p) + off + k);
      d[k] = t.x; d[k + 1] = t.y; d[k + 2] = t.z; d[k + 3] = t.w;
    }
    return;
  }
  if (st == 1 && dt == NKB_BF16 &&
      ((reinterpret_cast<uintptr_t>(static_cast<const __nv_bfloat16 *>(p) + off) & (2 * VEC - 1)) == 0)) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      const uint2 t = *reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(p) + off + k);
      d[k] = t.x << 16; d[k + 1] = t.x & 0xffff0000u; d[k + 2] = t.y << 16; d[k + 3] = t.y & 0xffff0000u;
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < VEC; ++k) d[k] = load_as_reg(p, off + k * st, dt);
}

template <int VEC>
__device__ __forceinline__ void store_run(void *p, int64_t off, int64_t st, int dt, const uint32_t (&v)[VEC]) {
  if (st == 1 && dt == NKB_F32 && ((reinterpret_cast<uintptr_t>(static_cast<float *>(p) + off) & 15) == 0)) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4)
      *reinterpret_cast<uint4 *>(static_cast<float *>(p) + off + k) = make_uint4(v[k], v[k + 1], v[k + 2], v[k + 3]);
    return;
  }
  if (st == 1 && dt == NKB_BF16 && ((reinterpret_cast<uintptr_t>(static_cast<__nv_bfloat16 *>(p) + off) & 7) == 0)) {
#pragma unroll
    for (int k = 0; k < VEC; k += 4) {
      __nv_bfloat162 a = __floats2bfloat162_rn(__uint_as_float(v[k]), __uint_as_float(v[k + 1]));
      __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(v[k + 2]), __uint_as_float(v[k + 3]));
      uint2 t;
      t.x = *reinterpret_cast<uint32_t *>(&a);
      t.y = *reinterpret_cast<uint32_t *>(&b);
      *reinterpret_cast<uint2 *>(static_cast<__nv_bfloat16 *>(p) + off + k) = t;
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < VEC; ++k) store_from_reg(p, off + k * st, dt, v[k]);
}

// Instruction flags of the row-run kernel, set at launch from the program:
// an operand equal to the previous instruction's destination is read from
// the accumulator (that result, still in registers); a result is written to
// the shared-memory register file only when a later instruction reads it
// from there or it is the output.  F_INPL: the instruction reads the
// accumulator as operand a and its opcode is applied in place (one test in
// the kernel instead of the opcode comparisons of inplace_op).
constexpr uint8_t F_A_ACC = 1, F_B_ACC = 2, F_C_ACC = 4, F_KEEP = 8, F_INPL = 16;
constexpr int kPre = 4;  // inputs whose run is loaded up front, all loads in flight together

template <typename IDX, int VEC>
__global__ void __launch_bounds__(256) ew_rows_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint32_t sreg[];
  const int T = blockDim.x;
  uint32_t *R = sreg + threadIdx.x;  // register (g, lane v) at R[(g * VEC + v) * T]
  const int last = p.rank - 1;
  const IDX inner = (IDX)p.shape[last];
  const IDX runs_per_row = inner / VEC;
  const IDX runs = (IDX)(p.n / VEC);
  for (IDX c = (IDX)blockIdx.x * blockDim.x + threadIdx.x; c < runs; c += (IDX)gridDim.x * blockDim.x) {
    // one axis (a collapsed dense view): no division per run
    const IDX row = last == 0 ? (IDX)0 : c / runs_per_row;
    const IDX col = (c - row * runs_per_row) * VEC;
    int64_t oo = p.out_off + (int64_t)col * p.out_strides[last];
    int64_t base[kMaxIn];
    for (int k = 0; k < p.n_in; ++k) base[k] = p.in_off[k] + (int64_t)col * p.in_strides[k][last];
    IDX rem = row;
    for (int d = last - 1; d >= 0; --d) {
      const IDX s = (IDX)p.shape[d];
      const IDX q = rem / s;
      const IDX id = rem - q * s;
      rem = q;
      oo += (int64_t)id * p.out_strides[d];
      for (int k = 0; k < p.n_in; ++k) base[k] += (int64_t)id * p.in_strides[k][d];
    }
    uint32_t acc[VEC];
    for (int pc = 0; pc < p.n_instr; ++pc) {
      const Instr I = p.prog[pc];
      uint32_t d[VEC];
      if (I.op == LD) {
        load_run<VEC>(p.in[I.a], base[I.a], p.in_strides[I.a][last], p.in_dtype[I.a], d);
      } else if (I.op == IOTA) {
        int64_t id = 0;
        if (I.a == last) {
          id = col;
        } else {
          IDX r2 = row;
          for (int dd = last - 1; dd >= 0; --dd) {
            const IDX s = (IDX)p.shape[dd];
            const IDX q = r2 / s;
            if (dd == I.a) id = r2 - q * s;
            r2 = q;
          }
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) d[v] = (uint32_t)(int32_t)(id + (I.a == last ? v : 0));
      } else if (I.pad & F_INPL) {
        uint32_t B[VEC];
        if (I.bimm) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = I.imm;
        } else if (I.pad & F_B_ACC) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = acc[v];
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = R[(I.b * VEC + v) * T];
        }
        compute_inplace<VEC>(I, acc, B);
        if (I.pad & F_KEEP) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) R[(I.dst * VEC + v) * T] = acc[v];
        }
        continue;
      } else {
        uint32_t A[VEC], B[VEC], C[VEC];
        if (I.pad & F_A_ACC) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) A[v] = acc[v];
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) A[v] = R[(I.a * VEC + v) * T];
        }
        if (I.bimm) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = I.imm;
        } else if (I.pad & F_B_ACC) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = acc[v];
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) B[v] = R[(I.b * VEC + v) * T];
        }
        if (I.op != SEL) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) C[v] = 0u;
        } else if (I.pad & F_C_ACC) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) C[v] = acc[v];
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) C[v] = R[(I.c * VEC + v) * T];
        }
        compute<VEC>(I, A, B, C, d);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = d[v];
      if (I.pad & F_KEEP) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) R[(I.dst * VEC + v) * T] = d[v];
      }
    }
    uint32_t o[VEC];
    if (p.prog[p.n_instr - 1].dst == p.out_reg) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = acc[v];
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = R[(p.out_reg * VEC + v) * T];
    }
    store_run<VEC>(p.out, oo, p.out_strides[last], p.out_dtype, o);
  }
}

// Sets the accumulator and keep flags of the row-run kernel (see F_A_ACC).
void set_row_flags(Params &p) {
  // the instruction whose result a register holds at each point, for KEEP
  int def[kRegs];
  for (int g = 0; g < kRegs; ++g) def[g] = -1;
  auto reads = [&](int j, int reg, uint8_t acc_flag) {
    Instr &J = p.prog[j];
    if (j > 0 && p.prog[j - 1].dst == reg) {
      J.pad |= acc_flag;
    } else if (def[reg] >= 0) {
      p.prog[def[reg]].pad |= F_KEEP;
    }
  };
  for (int j = 0; j < p.n_instr; ++j) {
    Instr &J = p.prog[j];
    J.pad = 0;
    if (J.op != LD && J.op != IOTA && J.op != CF && J.op != CI) {
      reads(j, J.a, F_A_ACC);
      if (!J.bimm) reads(j, J.b, F_B_ACC);
      if (J.op == SEL) reads(j, J.c, F_C_ACC);
    }
    def[J.dst] = j;
  }
  if (p.prog[p.n_instr - 1].dst != p.out_reg && def[p.out_reg] >= 0) p.prog[def[p.out_reg]].pad |= F_KEEP;
  for (int j = 0; j < p.n_instr; ++j)
    if ((p.prog[j].pad & F_A_ACC) && inplace_op(p.prog[j].op)) p.prog[j].pad |= F_INPL;
}

void parse(const Step &s, void *const *ptrs, Params &p);

// Step layout ("ew"):
//   ptrs:  out, in_0 .. in_{n_in-1}
//   ints:  n_in rank n_instr out_dtype out_reg contig n
//          shape[rank] out_off out_strides[rank]
//          per input: dtype off strides[rank]
//          per instr: op dst a b c imm_bits round(0/1 bf16/2 fp16) b_is_imm
int check(const Step &s) {
  if (s.ints.size() < 7) return fail(NKB_ERR_PLAN, "ew: short parameter list");
  const int64_t n_in = s.ints[0], rank = s.ints[1], n_instr = s.ints[2];
  if (n_in < 0 || n_in > kMaxIn) return fail(NKB_ERR_UNSUPPORTED, "ew: too many inputs");
  if (rank < 1 || rank > kMaxRank) return fail(NKB_ERR_UNSUPPORTED, "ew: rank out of range");
  if (n_instr < 1 || n_instr > kMaxInstr) return fail(NKB_ERR_UNSUPPORTED, "ew: program too long");
  const size_t want = 7 + rank + 1 + rank + n_in * (2 + rank) + n_instr * 8;
  if (s.ints.size() != want || s.buf_ids.size() != (size_t)(1 + n_in))
    return fail(NKB_ERR_PLAN, "ew: parameter count mismatch");
  const int64_t *q = s.ints.data() + 7 + rank + 1 + rank + n_in * (2 + rank);
  for (int i = 0; i < n_instr; ++i, q += 8) {
    if (q[1] >= kRegs || q[2] >= kRegs || q[3] >= kRegs || q[4] >= kRegs || q[1] < 0)
      return fail(NKB_ERR_PLAN, "ew: register index out of range");
    if (q[0] == LD && (q[2] < 0 || q[2] >= n_in)) return fail(NKB_ERR_PLAN, "ew: load of a missing input");
    if (q[0] == IOTA && (q[2] < 0 || q[2] >= rank)) return fail(NKB_ERR_PLAN, "ew: iota axis out of range");
  }
  if (s.ints[4] < 0 || s.ints[4] >= kRegs) return fail(NKB_ERR_PLAN, "ew: output register out of range");
  // compile the step's specialised kernel now, outside any graph capture
  Params p;
  parse(s, nullptr, p);
  if (p.n > 0 && p.shape[p.rank - 1] % 4 == 0) jit_prepare(p, s.ints);
  return NKB_OK;
}

// Fills the launch parameters from a checked step (device pointers from
// `ptrs`, or none when only the program and view are needed).
void parse(const Step &s, void *const *ptrs, Params &p) {
  memset(&p, 0, sizeof(p));
  const int64_t *q = s.ints.data();
  p.n_in = (int)q[0];
  p.rank = (int)q[1];
  p.n_instr = (int)q[2];
  p.out_dtype = (int)q[3];
  p.out_reg = (int)q[4];
  p.contig = (int)q[5];
  p.n = q[6];
  q += 7;
  for (int d = 0; d < p.rank; ++d) p.shape[d] = *q++;
  p.out_off = *q++;
  for (int d = 0; d < p.rank; ++d) p.out_strides[d] = *q++;
  p.out = ptrs ? ptrs[0] : nullptr;
  for (int k = 0; k < p.n_in; ++k) {
    p.in[k] = ptrs ? ptrs[1 + k] : nullptr;
    p.in_dtype[k] = (int)*q++;
    p.in_off[k] = *q++;
    for (int d = 0; d < p.rank; ++d) p.in_strides[k][d] = *q++;
  }
  for (int i = 0; i < p.n_instr; ++i) {
    Instr &I = p.prog[i];
    I.op = (uint8_t)q[0];
    I.dst = (uint8_t)q[1];
    I.a = (uint8_t)q[2];
    I.b = (uint8_t)q[3];
    I.c = (uint8_t)q[4];
    I.imm = (uint32_t)q[5];
    I.rnd = (uint8_t)q[6];
    I.bimm = (uint8_t)q[7];
    q += 8;
  }
}

int launch(const LaunchArgs &a) {
  Params p;
  parse(*a.step, a.ptrs, p);
  if (p.n == 0) return NKB_OK;
  if (p.shape[p.rank - 1] % 4 == 0) {
    bool launched = false;
    if (int st = jit_launch(p, a.step->ints, a.stream, a.device, &launched)) return st;
    if (launched) return NKB_OK;
  }
  const int threads = 256;
  int64_t blocks = (p.n + (int64_t)threads * kVec - 1) / ((int64_t)threads * kVec);
  const int64_t cap = (int64_t)num_sms(a.device) * 16;
  if (blocks > cap) blocks = cap;
  if (p.shape[p.rank - 1] % 4 == 0) {
    // 32-bit index math when the element count and every offset fit
    int64_t span = p.n;
    for (int k = 0; k < p.n_in; ++k) {
      int64_t hi = p.in_off[k];
      for (int d = 0; d < p.rank; ++d) hi += (p.shape[d] - 1) * (p.in_strides[k][d] < 0 ? 0 : p.in_strides[k][d]);
      span = span > hi ? span : hi;
    }
    int nregs = p.out_reg + 1;
    for (int i = 0; i < p.n_instr; ++i) {
      const Instr &I = p.prog[i];
      nregs = max(nregs, (int)I.dst + 1);
      if (I.op != LD && I.op != IOTA && I.op != CF && I.op != CI) {
        nregs = max(nregs, (int)I.a + 1);
        if (!I.bimm) nregs = max(nregs, (int)I.b + 1);
        if (I.op == SEL) nregs = max(nregs, (int)I.c + 1);
      }
    }
    set_row_flags(p);
    const bool v8 = p.shape[p.rank - 1] % 8 == 0;
    const int vec = v8 ? 8 : 4;
    const size_t smem = (size_t)nregs * vec * threads * 4;
    int64_t blocks2 = (p.n / vec + threads - 1) / threads;
    if (blocks2 > cap) blocks2 = cap;
    if (blocks2 < 1) blocks2 = 1;
    const bool small = span < INT32_MAX;
#define EW_ROWS(IDXT, V)                                                                                  \
  do {                                                                                                    \
    auto kfn = ew_rows_kernel<IDXT, V>;                                                                    \
    if (smem > 48 * 1024) NKB_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    kfn<<<(unsigned)blocks2, threads, smem, a.stream>>>(p);                                                \
  } while (0)
    if (small && v8) EW_ROWS(int32_t, 8);
    else if (small) EW_ROWS(int32_t, 4);
    else if (v8) EW_ROWS(int64_t, 8);
    else EW_ROWS(int64_t, 4);
#undef EW_ROWS
    return launch_status("ew_rows_kernel");
  }
  ew_kernel<<<(unsigned)blocks, threads, 0, a.stream>>>(p);
  return launch_status("ew_kernel");
}

}  // namespace ew

NKB_REGISTER_KERNEL("ew", ew::launch, ew::check);

// Compiles the specialised kernel of one "ew" step from its integer
// parameters (the step layout above), with NVRTC only: no device, no runtime
// initialisation.  *taken = 1 when the chain compiler took and compiled it.
extern "C" NKB_API int nkb_ew_compile_step(const int64_t *ints, size_t n_ints, int *taken) {
  if (!ints || !taken) return fail(NKB_ERR_INVALID, "NULL argument");
  *taken = 0;
  if (n_ints < 7 || ints[0] < 0 || ints[0] > ew::kMaxIn) return fail(NKB_ERR_PLAN, "ew: short or bad parameter list");
  Step s;
  s.kernel = "ew";
  s.ints.assign(ints, ints + n_ints);
  s.buf_ids.assign((size_t)ints[0] + 1, 0);
  s.buf_offsets.assign((size_t)ints[0] + 1, 0);
  if (int st = ew::check(s)) return st;
  ew::Params p;
  ew::parse(s, nullptr, p);
  if (p.n > 0 && p.shape[p.rank - 1] % 4 == 0) *taken = ew::jit_compiled(p, s.ints);
  return NKB_OK;
}

}  // namespace nkb
