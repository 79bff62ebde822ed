// C = A @ B for a few rows of A (M <= 16: the projections of a decode step,
// 8 token rows against a weight matrix), bf16 in, fp32 accumulation, bf16 out.
// Bound by the one read of B.  The rows of A, zero-padded to 16, are the A
// fragment of bf16 mma.sync m16n8k16; B (K x N, N contiguous, as the traced
// `x @ W` holds it) streams through a 6-stage cp.async ring of 32 k-rows x 256
// columns (16 KB, XOR-swizzled) and is read transposed by ldmatrix as the B
// fragment.  CTA (column block, k-range): four warps of 64 columns each;
// enough k-ranges for two CTAs per SM, their fp32 partial rows summed by
// gemm::splitk_reduce (one k-range: bf16 written directly).
#include "common.cuh"
#include "mma_sync.cuh"

namespace nkb {
namespace gemm {
int splitk_reduce(const float *ws, __nv_bfloat16 *C, int64_t M, int64_t N, int64_t ldc, int ks, cudaStream_t st,
                  int device);
}

namespace skinny {
using namespace mma;

constexpr int THREADS = 128;                 // four warps
constexpr int NT = 256;                      // output columns per CTA
constexpr int KT = 32;                       // k rows per stage
constexpr int STAGES = 6;
constexpr int STAGE_BYTES = KT * NT * 2;     // 16 KB
constexpr int MAX_KC = 1024;                 // k per CTA at most (A slice 16 x 1024 bf16 = 32 KB)

struct Params {
  const __nv_bfloat16 *A, *B;
  __nv_bfloat16 *C;
  float *ws;  // [ks][M][N] fp32 partials when ks > 1
  int64_t M, N, K, lda, ldb, ldc;
  int kc, ks;
  int b_pre;  // B is never written by an earlier step: its first stages load before pdl_wait
};

__global__ void __launch_bounds__(THREADS, 2) skinny_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *sA = smem;                      // [kc / 64][16 rows][128 B], swizzled
  uint8_t *sB = smem + 16 * p.kc * 2;      // STAGES x [32 rows][512 B], swizzled
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int64_t n0 = (int64_t)blockIdx.x * NT;
  const int s = blockIdx.y;
  const int64_t kbeg = (int64_t)s * p.kc, kend = min(p.K, kbeg + p.kc);
  const int nstage = (int)((kend - kbeg + KT - 1) / KT);

  auto load_stage = [&](int st, int buf) {
    const int64_t k0 = kbeg + (int64_t)st * KT;
    const uint32_t dst = smem_addr(sB + buf * STAGE_BYTES);
#pragma unroll
    for (int j = 0; j < KT * (NT / 8) / THREADS; ++j) {  // 8 chunks per thread
      const int idx = j * THREADS + tid, r = idx / (NT / 8), c = idx % (NT / 8);
      const int64_t k = k0 + r, n = n0 + c * 8;
      const bool ok = k < kend && n < p.N;
      const __nv_bfloat16 *src = p.B + (ok ? k * p.ldb + n : kbeg * p.ldb + n0);
      cp_async16(dst + swz(r, c, NT * 2), src, ok);
    }
  };
  // B stages that no earlier step writes (weights) start loading before the
  // wait on the previous kernel; everything else waits for it
  if (p.b_pre)
    for (int st = 0; st < STAGES - 1; ++st)
      if (st < nstage) load_stage(st, st);
  pdl_wait();
  pdl_trigger();
  // A slice: rows 0..15 (zero past M), k in [kbeg, kbeg + kc) (zero past K)
  const int cpr = p.kc / 8;  // 16-byte chunks per row of the slice
  for (int i = tid; i < 16 * cpr; i += THREADS) {
    const int r = i / cpr, c = i % cpr;
    const int64_t k = kbeg + c * 8;
    const bool ok = r < p.M && k < p.K;
    const __nv_bfloat16 *src = p.A + (ok ? (int64_t)r * p.lda + k : 0);
    cp_async16(smem_addr(sA) + (c / 8) * (16 * 128) + swz(r, c % 8, 128), src, ok);
  }
  // cp.async groups: 0 = A and stage 0 (with b_pre: the first STAGES - 1
  // stages), then one per remaining prologue stage (empty with b_pre)
  if (!p.b_pre && nstage > 0) load_stage(0, 0);
  cp_commit();
#pragma unroll
  for (int st = 1; st < STAGES - 1; ++st) {
    if (!p.b_pre && st < nstage) load_stage(st, st);
    cp_commit();
  }

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll 1
  for (int it = 0; it < nstage; ++it) {
    cp_wait<STAGES - 2>();
    __syncthreads();  // stage `it` landed for every thread; stage it-1 is consumed by every warp
    if (it + STAGES - 1 < nstage) load_stage(it + STAGES - 1, (it + STAGES - 1) % STAGES);
    cp_commit();
    const uint32_t bb = smem_addr(sB + (it % STAGES) * STAGE_BYTES);
#pragma unroll
    for (int kk = 0; kk < KT / 16; ++kk) {
      const int ki = it * (KT / 16) + kk;  // k-step of the slice
      uint32_t af[4];
      ldsm_x4(smem_addr(sA) + (ki / 4) * (16 * 128) + swz(lane % 16, (ki % 4) * 2 + lane / 16, 128), af[0], af[1],
              af[2], af[3]);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        ldsm_x4_t(bb + swz(r, warp * 8 + j + lane / 16, NT * 2), b0, b1, b2, b3);
        mma16816(o[j], af, b0, b1);
        mma16816(o[j + 1], af, b2, b3);
      }
    }
  }
  // rows lane / 4 and lane / 4 + 8, columns n0 + warp * 64 + j * 8 + (lane % 4) * 2 + {0, 1}
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t row = lane / 4 + h * 8;
    if (row >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t col = n0 + warp * 64 + j * 8 + (lane % 4) * 2;
      if (col >= p.N) continue;  // N % 8 == 0: the pair is whole
      if (p.ks == 1) {
        *reinterpret_cast<uint32_t *>(p.C + row * p.ldc + col) = pack2(o[j][2 * h], o[j][2 * h + 1]);
      } else {
        *reinterpret_cast<float2 *>(p.ws + ((int64_t)s * p.M + row) * p.N + col) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
      }
    }
  }
}

// "gemm_skinny": ptrs A B C WS; ints M N K lda ldb ldc kc [b_pre].  A (M x K, K contiguous),
// B (K x N, N contiguous), C (M x N) bf16; M <= 16; the planner sizes WS for
// ceil(K / kc) * M * N floats (unused with one k-range).  b_pre = 1 when no
// step of the plan writes B (a weight), so B may be read before the previous
// kernel has finished.
int check(const Step &st) {
  if (st.buf_ids.size() != 4 || (st.ints.size() != 7 && st.ints.size() != 8))
    return fail(NKB_ERR_PLAN, "gemm_skinny: bad parameters");
  const auto &q = st.ints;
  if (q[0] < 0 || q[0] > 16) return fail(NKB_ERR_UNSUPPORTED, "gemm_skinny: at most 16 rows");
  if (q[2] % 8 || q[1] % 8 || q[3] % 8 || q[4] % 8 || q[5] % 2)
    return fail(NKB_ERR_UNSUPPORTED, "gemm_skinny: K, N and row strides must be multiples of 8 elements");
  if (q[6] < 64 || q[6] % 64 || q[6] > MAX_KC) return fail(NKB_ERR_PLAN, "gemm_skinny: k per CTA out of range");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  Params p;
  p.A = static_cast<const __nv_bfloat16 *>(a.ptrs[0]);
  p.B = static_cast<const __nv_bfloat16 *>(a.ptrs[1]);
  p.C = static_cast<__nv_bfloat16 *>(a.ptrs[2]);
  p.ws = static_cast<float *>(a.ptrs[3]);
  p.M = q[0];
  p.N = q[1];
  p.K = q[2];
  p.lda = q[3];
  p.ldb = q[4];
  p.ldc = q[5];
  p.kc = (int)q[6];
  p.b_pre = q.size() > 7 ? (int)q[7] : 0;
  if (p.M == 0 || p.N == 0) return NKB_OK;
  if (p.K == 0) return fail(NKB_ERR_UNSUPPORTED, "gemm_skinny: K == 0");
  p.ks = (int)((p.K + p.kc - 1) / p.kc);
  if (((reinterpret_cast<uintptr_t>(p.A) | reinterpret_cast<uintptr_t>(p.B)) & 15) ||
      (reinterpret_cast<uintptr_t>(p.C) & 3) || (p.ks > 1 && (reinterpret_cast<uintptr_t>(p.ws) & 7)))
    return fail(NKB_ERR_UNSUPPORTED, "gemm_skinny: operands not aligned for 16-byte copies");
  const int smem = 16 * p.kc * 2 + STAGES * STAGE_BYTES;
  static ContextOnce attr_set;
  if (int s = attr_set.run(a.device, []() -> int {
        NKB_CUDA_TRY(cudaFuncSetAttribute(skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          16 * MAX_KC * 2 + STAGES * STAGE_BYTES));
        return NKB_OK;
      }))
    return s;
  dim3 grid((unsigned)((p.N + NT - 1) / NT), (unsigned)p.ks);
  launch_pdl(a.pdl, skinny_kernel, grid, THREADS, smem, a.stream, p);
  if (int e = launch_status("skinny_kernel")) return e;
  if (p.ks > 1) return gemm::splitk_reduce(p.ws, p.C, p.M, p.N, p.ldc, p.ks, a.stream, a.device);
  return NKB_OK;
}

}  // namespace skinny

NKB_REGISTER_KERNEL("gemm_skinny", skinny::launch, skinny::check);

}  // namespace nkb
