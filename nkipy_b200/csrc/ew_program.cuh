// Program format of the fused elementwise kernels: the register program a
// step carries (opcodes, instruction layout) and the launch parameters.  Shared
// by the interpreter (k_elementwise.cu) and the chain compiler (ew_jit.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace nkb {
namespace ew {

constexpr int kMaxIn = 8;
constexpr int kMaxRank = 6;
constexpr int kMaxInstr = 64;
constexpr int kRegs = 24;
constexpr int kVec = 4;

enum Opcode : uint8_t {
  NOP = 0, LD = 1, CF = 2, CI = 3, IOTA = 4,
  FADD = 10, FSUB, FMUL, FDIV, FPOW, FMAX, FMIN, FATAN2, FREM,
  FNEG = 20, FABS, FEXP, FLOG, FSQRT, FRSQRT, FTANH, FSIN, FCOS, FFLOOR, FCEIL, FSIGN, RBF, RF16, FRCP,
  FEQ = 40, FNE, FLT, FLE, FGT, FGE,
  IADD = 50, ISUB, IMUL, IDIV, IMAX, IMIN, IAND, IOR, IXOR, IREM,
  ISHL = 64, ISHR = 65,
  INEG = 60, IABS, INOT, ISIGN,
  IEQ = 70, INE, ILT, ILE, IGT, IGE, ULT, ULE, UGT, UGE, UDIV, UMAX, UMIN, UREM,
  SEL = 90,
  F2I = 100, I2F, U2F, F2U, INZ, FNZ
};

struct Instr {
  uint8_t op, dst, a, b, c;
  uint8_t rnd;   // round the result: 1 = to bf16, 2 = to fp16
  uint8_t bimm;  // 1 = operand b is the immediate `imm`
  uint8_t pad;
  uint32_t imm;
};

struct Params {
  int n_in, rank, n_instr, out_dtype, out_reg, contig;
  int64_t n;
  int64_t shape[kMaxRank];
  void *out;
  int64_t out_off;
  int64_t out_strides[kMaxRank];
  const void *in[kMaxIn];
  int in_dtype[kMaxIn];
  int64_t in_off[kMaxIn];
  int64_t in_strides[kMaxIn][kMaxRank];
  Instr prog[kMaxInstr];
};

// The chain compiler (ew_jit.cu).  jit_prepare compiles the kernel specialised
// to a step's program, shapes and strides (once per distinct step) and loads it
// in the current context; it returns 1 when the step will run on it.
// jit_launch launches that kernel and sets *launched, or leaves the step to the
// interpreter (*launched false: compiler unavailable or disabled, or the module
// not loaded in this context while a graph is being captured); it returns a
// status.
// `ints` are the step's integer parameters (from which `p` was parsed): the
// key of the per-step kernel cache.
int jit_prepare(const Params &p, const std::vector<int64_t> &ints);
int jit_launch(const Params &p, const std::vector<int64_t> &ints, cudaStream_t stream, int device, bool *launched);
// 1 when the step's kernel is compiled (compiling it now if needed; no device
// is used), 0 when the compiler does not take the step or cannot compile it.
int jit_compiled(const Params &p, const std::vector<int64_t> &ints);

}  // namespace ew
}  // namespace nkb
