// Fused causal attention (prefill): the traced composition
//   scores = q @ k^T ; scores / sqrt(d) ; + causal mask ; softmax ; @ v
// of examples/models/qwen3_embedding/kernels/attention.py:85-95 and
// examples/models/qwen3/kernels/attention.py:119-140, computed without
// materialising the S x S score matrix (online softmax, fp32 statistics).
//
// GQA: query head h reads kv head h / (H / Hkv), so the traced np.repeat of
// k and v never reaches memory.  Q, K, V and O are strided views
// (batch, head, position strides in elements, head_dim contiguous), so the
// transposes around the attention are free as well.
//
// Tiling: one CTA = 128 query rows of one (batch, head), 8 warps x 16 rows;
// key/value tiles of 64 rows double-buffered in shared memory with
// cp.async; bf16 mma.sync m16n8k16 with fp32 accumulation; P stays in
// registers between the two products.  Shared-memory rows are XOR-swizzled
// at 16-byte granularity so ldmatrix reads are bank-conflict free.  Causal
// CTAs run longest-first.

#include "common.cuh"

namespace nkb {

bool fa_tc_eligible(int D, int64_t qs, int64_t ks, int64_t vs, int64_t os);
int fa_tc_launch(const void *q, const void *k, const void *v, void *o, int B, int H, int Hkv, int Sq, int Skv,
                 int causal, float scale, const int64_t *qst, const int64_t *kst, const int64_t *vst,
                 const int64_t *ost, cudaStream_t st, int device);

namespace attn {

constexpr int BM = 128, BN = 64, WARPS = 8;

struct Params {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16 *o;
  int B, H, Hkv, Sq, Skv, causal;
  int64_t qb, qh, qs, kb, kh, ks, vb, vh, vs, ob, oh, os;
  float scale_log2;  // softmax scale * log2(e)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  // byte offset of 16-byte chunk `chunk` of row `row` in a [rows][D] bf16 tile
  return row * (D * 2) + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool pred) {
  const int n = pred ? 16 : 0;  // zero-fill rows outside the sequence
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

template <int D>
__device__ __forceinline__ void load_tile(uint8_t *smem, const __nv_bfloat16 *base, int64_t row_stride, int row0,
                                          int rows, int limit) {
  constexpr int CHUNKS = D / 8;
  const uint32_t s0 = smem_u32(smem);
  for (int i = threadIdx.x; i < rows * CHUNKS; i += WARPS * 32) {
    const int r = i / CHUNKS, c = i % CHUNKS;
    const int gr = row0 + r;
    const bool ok = gr < limit;
    const __nv_bfloat16 *src = base + (int64_t)(ok ? gr : 0) * row_stride + c * 8;
    cp_async16(s0 + swz<D>(r, c), src, ok);
  }
}

template <int D>
__global__ void __launch_bounds__(WARPS * 32, 1) flash_fwd_kernel(const __grid_constant__ Params p) {
  constexpr int KSTEPS = D / 16;   // k-steps over head_dim
  constexpr int DTILES = D / 8;    // n-tiles of the output
  constexpr int NTILES = BN / 8;   // n-tiles of the score block
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *sQ = smem;
  uint8_t *sK = smem + BM * D * 2;
  uint8_t *sV = sK + 2 * BN * D * 2;

  const int n_qt = (p.Sq + BM - 1) / BM;
  const int qt = p.causal ? (n_qt - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = qt * BM;

  const __nv_bfloat16 *Qb = p.q + b * p.qb + h * p.qh;
  const __nv_bfloat16 *Kb = p.k + b * p.kb + hk * p.kh;
  const __nv_bfloat16 *Vb = p.v + b * p.vb + hk * p.vh;

  // causal: keys needed up to the last query row of this tile
  const int kv_end = p.causal ? min(p.Skv, q0 + BM + (p.Skv - p.Sq)) : p.Skv;
  const int n_kt = (kv_end + BN - 1) / BN;

  load_tile<D>(sQ, Qb, p.qs, q0, BM, p.Sq);
  cp_commit();
  if (n_kt > 0) {
    load_tile<D>(sK, Kb, p.ks, 0, BN, p.Skv);
    load_tile<D>(sV, Vb, p.vs, 0, BN, p.Skv);
  }
  cp_commit();

  // Q fragments for this warp's 16 rows, kept in registers
  uint32_t qf[KSTEPS][4];
  cp_wait<1>();
  __syncthreads();
  {
    const uint32_t s0 = smem_u32(sQ);
    const int r = warp * 16 + (lane % 16);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      ldsm_x4(s0 + swz<D>(r, kk * 2 + lane / 16), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float o[DTILES][4];
#pragma unroll
  for (int j = 0; j < DTILES; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int row_a = q0 + warp * 16 + lane / 4;  // rows owned by this thread: row_a, row_a + 8
  const int diag_shift = p.Skv - p.Sq;

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) {
      load_tile<D>(sK + (buf ^ 1) * BN * D * 2, Kb, p.ks, (kt + 1) * BN, BN, p.Skv);
      load_tile<D>(sV + (buf ^ 1) * BN * D * 2, Vb, p.vs, (kt + 1) * BN, BN, p.Skv);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();

    const uint32_t kbase = smem_u32(sK + buf * BN * D * 2);
    const uint32_t vbase = smem_u32(sV + buf * BN * D * 2);
    float s[NTILES][4];
#pragma unroll
    for (int j = 0; j < NTILES; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int j = 0; j < NTILES; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = j * 8 + (lane % 8) + (lane / 16) * 8;
        ldsm_x4(kbase + swz<D>(r, kk * 2 + (lane / 8) % 2), b0, b1, b2, b3);
        mma16816(s[j], qf[kk], b0, b1);
        mma16816(s[j + 1], qf[kk], b2, b3);
      }
    }
    // scale, causal mask, online softmax
    const int k0 = kt * BN;
    const bool need_mask = p.causal && (k0 + BN - 1 > q0 + warp * 16 + diag_shift) ;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < NTILES; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = k0 + j * 8 + (lane % 4) * 2 + (e & 1);
        const int row = row_a + (e >> 1) * 8;
        float v = s[j][e] * p.scale_log2;
        if (col >= p.Skv || (need_mask && col > row + diag_shift)) v = -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      alpha[i] = (mx[i] == -INFINITY) ? 1.f : exp2f(m_r[i] - mx[i]);
      m_r[i] = mx[i];
    }
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int j = 0; j < NTILES; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mrow = m_r[e >> 1];
        const float pv = (mrow == -INFINITY) ? 0.f : exp2f(s[j][e] - mrow);
        s[j][e] = pv;
        rs[e >> 1] += pv;
      }
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      pf[kk][0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pf[kk][1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pf[kk][2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pf[kk][3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) l_r[i] = l_r[i] * alpha[i] + rs[i];
#pragma unroll
    for (int j = 0; j < DTILES; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < DTILES; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        ldsm_x4_t(vbase + swz<D>(r, j + lane / 16), b0, b1, b2, b3);
        mma16816(o[j], pf[kk], b0, b1);
        mma16816(o[j + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();
  }

  // finish the row sums across the quad, normalise, store bf16
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
  __nv_bfloat16 *Ob = p.o + b * p.ob + h * p.oh;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int row = row_a + i * 8;
    if (row >= p.Sq) continue;
    const float inv = l_r[i] > 0.f ? 1.f / l_r[i] : 0.f;
    __nv_bfloat16 *orow = Ob + (int64_t)row * p.os;
#pragma unroll
    for (int j = 0; j < DTILES; ++j) {
      const int col = j * 8 + (lane % 4) * 2;
      *reinterpret_cast<uint32_t *>(orow + col) = pack_bf16(o[j][2 * i] * inv, o[j][2 * i + 1] * inv);
    }
  }
}

template <int D>
int launch_d(const Params &p, cudaStream_t st) {
  const int smem = (BM + 4 * BN) * D * 2;
  static ContextOnce attr;
  int dev = 0;
  NKB_CUDA_TRY(cudaGetDevice(&dev));
  if (int s = attr.run(dev, [&]() -> int {
        NKB_CUDA_TRY(cudaFuncSetAttribute(flash_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return NKB_OK;
      }))
    return s;
  dim3 grid((p.Sq + BM - 1) / BM, p.B * p.H);
  flash_fwd_kernel<D><<<grid, WARPS * 32, smem, st>>>(p);
  return launch_status("flash_fwd_kernel");
}

// "flash_attn": ptrs q k v o; ints B H Hkv Sq Skv D causal qb qh qs kb kh ks vb vh vs ob oh os; floats scale
int check(const Step &s) {
  if (s.buf_ids.size() != 4 || s.ints.size() != 19 || s.floats.size() != 1)
    return fail(NKB_ERR_PLAN, "flash_attn: bad parameters");
  const int64_t D = s.ints[5], H = s.ints[1], Hkv = s.ints[2];
  if (D != 64 && D != 128) return fail(NKB_ERR_UNSUPPORTED, "flash_attn: head_dim must be 64 or 128");
  if (Hkv <= 0 || H % Hkv) return fail(NKB_ERR_UNSUPPORTED, "flash_attn: heads must be a multiple of kv heads");
  for (int i = 7; i < 19; ++i)
    if (s.ints[i] % 8) return fail(NKB_ERR_UNSUPPORTED, "flash_attn: strides must be multiples of 8 elements");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  Params p;
  p.q = static_cast<const __nv_bfloat16 *>(a.ptrs[0]);
  p.k = static_cast<const __nv_bfloat16 *>(a.ptrs[1]);
  p.v = static_cast<const __nv_bfloat16 *>(a.ptrs[2]);
  p.o = static_cast<__nv_bfloat16 *>(a.ptrs[3]);
  p.B = (int)q[0];
  p.H = (int)q[1];
  p.Hkv = (int)q[2];
  p.Sq = (int)q[3];
  p.Skv = (int)q[4];
  p.causal = (int)q[6];
  p.qb = q[7];
  p.qh = q[8];
  p.qs = q[9];
  p.kb = q[10];
  p.kh = q[11];
  p.ks = q[12];
  p.vb = q[13];
  p.vh = q[14];
  p.vs = q[15];
  p.ob = q[16];
  p.oh = q[17];
  p.os = q[18];
  p.scale_log2 = a.step->floats[0] * 1.4426950408889634f;
  for (int i = 0; i < 4; ++i)
    if (reinterpret_cast<uintptr_t>(a.ptrs[i]) & 15) return fail(NKB_ERR_UNSUPPORTED, "flash_attn: unaligned base");
  if (p.B == 0 || p.H == 0 || p.Sq == 0) return NKB_OK;
  // head_dim 128: tcgen05 kernel (k_flash_sm100.cu); head_dim 64: mma.sync kernel below
  if (fa_tc_eligible((int)q[5], p.qs, p.ks, p.vs, p.os))
    return fa_tc_launch(p.q, p.k, p.v, p.o, p.B, p.H, p.Hkv, p.Sq, p.Skv, p.causal, a.step->floats[0], &q[7], &q[10],
                        &q[13], &q[16], a.stream, a.device);
  return q[5] == 128 ? launch_d<128>(p, a.stream) : launch_d<64>(p, a.stream);
}

}  // namespace attn

NKB_REGISTER_KERNEL("flash_attn", attn::launch, attn::check);

}  // namespace nkb
