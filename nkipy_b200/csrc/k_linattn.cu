// Chunked causal linear attention (feature map elu + 1, chunk 64, fp32 state):
//   phi = elu + 1;  S_c = sum_{chunks < c} phi(K)^T V,  z_c = sum_{chunks < c} phi(K)
//   out_c = (tril(phi(Q_c) phi(K_c)^T) V_c + phi(Q_c) S_c)
//           / (rowsum(tril(phi(Q_c) phi(K_c)^T)) + phi(Q_c) . z_c)
// -- the kernel body nkipy_b200/workloads.py:chunked_linear_attention_kernel,
// whose per-step state update follows examples/linear_attention/deltanet.py.
//
// One CTA per (batch*head, segment of the sequence); 8 warps.
//   phase 0 (state): each segment's sum of phi(K)^T V and of phi(K) over its
//                    chunks -> workspace (fp32, D x D + D per segment);
//   scan:             per head, the segment states become exclusive prefixes;
//   phase 1 (output): the CTA seeds its running state with its segment's
//                    prefix, then walks its chunks: intra-chunk masked scores,
//                    the state product, the normaliser, and the state update.
// Chunks of q/k/v are double-buffered in shared memory with cp.async; the
// feature map is applied in place; products use bf16 mma.sync m16n8k16 with
// fp32 accumulation; the running state S is kept in fp32 registers (16 rows of
// S per warp) and mirrored to shared memory in bf16 as the operand of
// phi(Q) S.  The workspace is the only memory beyond inputs and output.

#include <mutex>

#include "common.cuh"

namespace nkb {
namespace linattn {

constexpr int C = 64, D = 128, WARPS = 8, THREADS = WARPS * 32;
constexpr int TILE = C * D * 2;  // bytes of one bf16 chunk tile

struct Params {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16 *o;
  float *ws;  // [B*H][G][D*D + D]
  int BH, H, T, G, chunks_per_seg, phase;
  int64_t qb, qh, qs, kb, kh, ks, vb, vh, vs, ob, oh, os;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
template <int W>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return row * (W * 2) + ((chunk ^ (row & 7)) << 4);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
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

// one chunk (C rows x D) of a strided (b, h, t, d) tensor into a swizzled tile
__device__ __forceinline__ void load_chunk(uint8_t *tile, const __nv_bfloat16 *base, int64_t row_stride, int t0) {
  const uint32_t s0 = smem_u32(tile);
  for (int i = threadIdx.x; i < C * (D / 8); i += THREADS) {
    const int r = i / (D / 8), c = i % (D / 8);
    cp_async16(s0 + swz<D>(r, c), base + (int64_t)(t0 + r) * row_stride + c * 8);
  }
}

// phi = elu + 1 in place on a bf16 tile; optionally accumulate column sums of phi
__device__ __forceinline__ void feature_map(uint8_t *tile, float *colsum) {
  const int col = threadIdx.x % D;
  const int r0 = (threadIdx.x / D) * (C / (THREADS / D));
  float acc = 0.f;
  for (int r = r0; r < r0 + C / (THREADS / D); ++r) {
    __nv_bfloat16 *p = reinterpret_cast<__nv_bfloat16 *>(tile + swz<D>(r, col / 8)) + (col % 8);
    const float x = __bfloat162float(*p);
    const float f = x > 0.f ? x + 1.f : expf(x);
    const __nv_bfloat16 fb = __float2bfloat16_rn(f);
    *p = fb;
    acc += __bfloat162float(fb);
  }
  if (colsum) atomicAdd(&colsum[col], acc);
}

__global__ void __launch_bounds__(THREADS, 1) linattn_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  // [stage][q,k,v] raw/feature-mapped chunks, then S (bf16), P (bf16), small vectors
  uint8_t *stage0 = smem;
  uint8_t *sS = smem + 2 * 3 * TILE;
  uint8_t *sP = sS + D * D * 2;
  float *sZ = reinterpret_cast<float *>(sP + C * C * 2);  // running key-sum (prefix)
  float *sZadd = sZ + D;                                 // this chunk's key column sums
  float *sRow = sZadd + D;                               // [2][C] partial row sums of masked scores
  float *sDen = sRow + 2 * C;                            // [C]

  const int bh = blockIdx.y, seg = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const __nv_bfloat16 *Qb = p.q + b * p.qb + h * p.qh;
  const __nv_bfloat16 *Kb = p.k + b * p.kb + h * p.kh;
  const __nv_bfloat16 *Vb = p.v + b * p.vb + h * p.vh;
  float *ws = p.ws + (int64_t)bh * p.G * (D * D + D);
  const bool out_phase = p.phase == 1;

  // running state: warp w owns S rows [16w, 16w+16), all D columns
  float S[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.f;
  const int srow = warp * 16 + lane / 4;
  for (int i = threadIdx.x; i < D; i += THREADS) sZ[i] = 0.f;
  if (out_phase && seg > 0) {
    // seed with the exclusive prefix of the earlier segments of this head
    const float *w = ws + (int64_t)seg * (D * D + D);
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int col = j * 8 + (lane % 4) * 2;
      S[j][0] = w[srow * D + col];
      S[j][1] = w[srow * D + col + 1];
      S[j][2] = w[(srow + 8) * D + col];
      S[j][3] = w[(srow + 8) * D + col + 1];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += THREADS) sZ[i] = w[D * D + i];
  }
  // bf16 mirror of S for phi(Q) S
  auto publish_S = [&]() {
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int col = j * 8 + (lane % 4) * 2;
      *reinterpret_cast<uint32_t *>(sS + swz<D>(srow, col / 8) + (col % 8) * 2) = pack_bf16(S[j][0], S[j][1]);
      *reinterpret_cast<uint32_t *>(sS + swz<D>(srow + 8, col / 8) + (col % 8) * 2) = pack_bf16(S[j][2], S[j][3]);
    }
  };
  if (out_phase) publish_S();

  const int c0 = seg * p.chunks_per_seg;
  const int n = min(p.chunks_per_seg, p.T / C - c0);
  auto issue = [&](int ci, int stg) {
    uint8_t *base = stage0 + stg * 3 * TILE;
    const int t0 = (c0 + ci) * C;
    if (out_phase) load_chunk(base, Qb, p.qs, t0);
    load_chunk(base + TILE, Kb, p.ks, t0);
    load_chunk(base + 2 * TILE, Vb, p.vs, t0);
  };
  issue(0, 0);
  cp_commit();

  for (int ci = 0; ci < n; ++ci) {
    const int stg = ci & 1;
    if (ci + 1 < n) issue(ci + 1, stg ^ 1);
    cp_commit();
    cp_wait<1>();
    for (int i = threadIdx.x; i < D; i += THREADS) sZadd[i] = 0.f;
    __syncthreads();
    uint8_t *tq = stage0 + stg * 3 * TILE;
    uint8_t *tk = tq + TILE;
    uint8_t *tv = tk + TILE;
    if (out_phase) feature_map(tq, nullptr);
    feature_map(tk, sZadd);
    __syncthreads();

    if (out_phase) {
      // ---- masked scores P = tril(phi(Q) phi(K)^T): warp -> rows 16*(w%4), cols 32*(w/4)
      const int mr = (warp % 4) * 16, nc = (warp / 4) * 32;
      float sc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
      const uint32_t qa = smem_u32(tq), ka = smem_u32(tk);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(qa + swz<D>(mr + (lane % 16), kk * 2 + lane / 16), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = nc + j * 8 + (lane % 8) + (lane / 16) * 8;
          ldsm_x4(ka + swz<D>(r, kk * 2 + (lane / 8) % 2), b0, b1, b2, b3);
          mma16816(sc[j], a, b0, b1);
          mma16816(sc[j + 1], a, b2, b3);
        }
      }
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = mr + lane / 4 + (e >> 1) * 8;
          const int col = nc + j * 8 + (lane % 4) * 2 + (e & 1);
          if (col > row) sc[j][e] = 0.f;
          rs[e >> 1] += sc[j][e];
        }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
        rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      }
      if (lane % 4 == 0) {
        sRow[(warp / 4) * C + mr + lane / 4] = rs[0];
        sRow[(warp / 4) * C + mr + lane / 4 + 8] = rs[1];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = nc + j * 8 + (lane % 4) * 2;
        const int row = mr + lane / 4;
        *reinterpret_cast<uint32_t *>(sP + swz<C>(row, col / 8) + (col % 8) * 2) = pack_bf16(sc[j][0], sc[j][1]);
        *reinterpret_cast<uint32_t *>(sP + swz<C>(row + 8, col / 8) + (col % 8) * 2) = pack_bf16(sc[j][2], sc[j][3]);
      }
      __syncthreads();
      // ---- normaliser: rowsum + phi(Q) . z   (warp -> 8 rows)
      for (int rr = 0; rr < C / WARPS; ++rr) {
        const int row = warp * (C / WARPS) + rr;
        float acc = 0.f;
#pragma unroll
        for (int q4 = 0; q4 < D / 32; ++q4) {
          const int col = q4 * 32 + lane;
          const float x = __bfloat162float(
              *(reinterpret_cast<const __nv_bfloat16 *>(tq + swz<D>(row, col / 8)) + (col % 8)));
          acc += x * sZ[col];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) sDen[row] = acc + sRow[row] + sRow[C + row];
      }
      // ---- numerator: P V + phi(Q) S   (warp -> rows 16*(w%4), cols 64*(w/4))
      const int oc = (warp / 4) * 64;
      float num[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) num[j][0] = num[j][1] = num[j][2] = num[j][3] = 0.f;
      const uint32_t pa = smem_u32(sP), va = smem_u32(tv), sa = smem_u32(sS);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(pa + swz<C>(mr + (lane % 16), kk * 2 + lane / 16), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
          ldsm_x4_t(va + swz<D>(r, oc / 8 + j + lane / 16), b0, b1, b2, b3);
          mma16816(num[j], a, b0, b1);
          mma16816(num[j + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(qa + swz<D>(mr + (lane % 16), kk * 2 + lane / 16), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
          ldsm_x4_t(sa + swz<D>(r, oc / 8 + j + lane / 16), b0, b1, b2, b3);
          mma16816(num[j], a, b0, b1);
          mma16816(num[j + 1], a, b2, b3);
        }
      }
      __syncthreads();  // sDen complete
      const int t0 = (c0 + ci) * C;
      __nv_bfloat16 *Ob = p.o + b * p.ob + h * p.oh;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int row = mr + lane / 4 + i * 8;
        const float inv = 1.f / sDen[row];
        __nv_bfloat16 *orow = Ob + (int64_t)(t0 + row) * p.os;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = oc + j * 8 + (lane % 4) * 2;
          *reinterpret_cast<uint32_t *>(orow + col) = pack_bf16(num[j][2 * i] * inv, num[j][2 * i + 1] * inv);
        }
      }
    }

    // ---- state update S += phi(K)^T V  (warp -> S rows 16w)
    {
      const uint32_t ka = smem_u32(tk), va = smem_u32(tv);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t a[4];
        const int tok = kk * 16 + (lane % 8) + (lane / 16) * 8;
        const int dch = (warp * 16) / 8 + (lane / 8) % 2;
        ldsm_x4_t(ka + swz<D>(tok, dch), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int j = 0; j < D / 8; j += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
          ldsm_x4_t(va + swz<D>(r, j + lane / 16), b0, b1, b2, b3);
          mma16816(S[j], a, b0, b1);
          mma16816(S[j + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += THREADS) sZ[i] += sZadd[i];
    if (out_phase) publish_S();
    __syncthreads();
  }

  if (!out_phase) {
    float *w = ws + (int64_t)seg * (D * D + D);
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int col = j * 8 + (lane % 4) * 2;
      w[srow * D + col] = S[j][0];
      w[srow * D + col + 1] = S[j][1];
      w[(srow + 8) * D + col] = S[j][2];
      w[(srow + 8) * D + col + 1] = S[j][3];
    }
    for (int i = threadIdx.x; i < D; i += THREADS) w[D * D + i] = sZ[i];
  }
}

constexpr int SMEM = 2 * 3 * TILE + D * D * 2 + C * C * 2 + (2 * D + 3 * C) * 4;
constexpr int SEG_CHUNKS = 16;  // chunks (of 64 tokens) per segment

// per head: segment states -> exclusive prefixes over the segments, in place
__global__ void __launch_bounds__(256) linattn_scan_kernel(float *ws, int G) {
  float *w = ws + (int64_t)blockIdx.x * G * (D * D + D);
  for (int i = threadIdx.x; i < D * D + D; i += blockDim.x) {
    float run = 0.f;
    for (int g = 0; g < G; ++g) {
      const float x = w[(int64_t)g * (D * D + D) + i];
      w[(int64_t)g * (D * D + D) + i] = run;
      run += x;
    }
  }
}

int run(const Params &base, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    NKB_CUDA_TRY(cudaFuncSetAttribute(linattn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr = true;
  }
  dim3 grid(base.G, base.BH);
  Params p = base;
  if (p.G > 1) {
    p.phase = 0;
    linattn_kernel<<<grid, THREADS, SMEM, st>>>(p);
    if (int s = launch_status("linattn_kernel(state)")) return s;
    linattn_scan_kernel<<<p.BH, 256, 0, st>>>(p.ws, p.G);
    if (int s = launch_status("linattn_scan_kernel")) return s;
  }
  p.phase = 1;
  linattn_kernel<<<grid, THREADS, SMEM, st>>>(p);
  return launch_status("linattn_kernel(output)");
}

// segments per head: SEG_CHUNKS chunks each (the last one may be shorter)
int pick_segments(int BH, int T, int device) {
  (void)BH;
  (void)device;
  const int chunks = T / C;
  return chunks <= SEG_CHUNKS ? 1 : (chunks + SEG_CHUNKS - 1) / SEG_CHUNKS;
}

size_t workspace_bytes(int BH, int G) { return (size_t)BH * G * (D * D + D) * sizeof(float); }

// "linattn": ptrs q k v o ws; ints B H T Dh G qb qh qs kb kh ks vb vh vs ob oh os
int check(const Step &s) {
  if (s.buf_ids.size() != 5 || s.ints.size() != 17) return fail(NKB_ERR_PLAN, "linattn: bad parameters");
  if (s.ints[3] != D) return fail(NKB_ERR_UNSUPPORTED, "linattn: head_dim must be 128");
  if (s.ints[2] % C) return fail(NKB_ERR_UNSUPPORTED, "linattn: length must be a multiple of 64");
  const int64_t chunks = s.ints[2] / C;
  const int64_t G = chunks <= SEG_CHUNKS ? 1 : (chunks + SEG_CHUNKS - 1) / SEG_CHUNKS;
  if (s.ints[4] != G) return fail(NKB_ERR_PLAN, "linattn: segment count does not match the kernel's segmentation");
  for (int i = 5; i < 17; ++i)
    if (s.ints[i] % 8) return fail(NKB_ERR_UNSUPPORTED, "linattn: strides must be multiples of 8");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  Params p;
  p.q = static_cast<const __nv_bfloat16 *>(a.ptrs[0]);
  p.k = static_cast<const __nv_bfloat16 *>(a.ptrs[1]);
  p.v = static_cast<const __nv_bfloat16 *>(a.ptrs[2]);
  p.o = static_cast<__nv_bfloat16 *>(a.ptrs[3]);
  p.ws = static_cast<float *>(a.ptrs[4]);
  const int B = (int)q[0];
  p.H = (int)q[1];
  p.BH = B * p.H;
  p.T = (int)q[2];
  p.G = (int)q[4];
  p.chunks_per_seg = p.G > 1 ? SEG_CHUNKS : p.T / C;
  p.qb = q[5]; p.qh = q[6]; p.qs = q[7];
  p.kb = q[8]; p.kh = q[9]; p.ks = q[10];
  p.vb = q[11]; p.vh = q[12]; p.vs = q[13];
  p.ob = q[14]; p.oh = q[15]; p.os = q[16];
  for (int i = 0; i < 4; ++i)
    if (reinterpret_cast<uintptr_t>(a.ptrs[i]) & 15) return fail(NKB_ERR_UNSUPPORTED, "linattn: unaligned base");
  if (p.BH == 0 || p.T == 0) return NKB_OK;
  return run(p, a.stream);
}

}  // namespace linattn

NKB_REGISTER_KERNEL("linattn", linattn::launch, linattn::check);

int linattn_segments(int BH, int T, int device) { return linattn::pick_segments(BH, T, device); }
size_t linattn_workspace_bytes(int BH, int G) { return linattn::workspace_bytes(BH, G); }

// ---------------------------------------------------------------------------
// Allocation-free variant
// ---------------------------------------------------------------------------
// The planned path gets its segment-state workspace from the plan's scratch
// arena, which the runtime allocates when the plan is loaded.  Some callers
// cannot allocate device memory at the point where they run this kernel: a
// host process that has handed the whole GPU to its own caching allocator up
// front, or a latency-critical loop in which a cudaMalloc/cudaFree could
// block or synchronise the device.  For them the workspace lives in a fixed,
// file-scope device array of NKB_LINATTN_SCRATCH_BYTES: every GPU that loads
// this library holds it until the process exits, and every call shares it.
namespace linattn {

static __device__ __align__(256) unsigned char g_scratch[NKB_LINATTN_SCRATCH_BYTES];

static void *g_scratch_addr[64];
static std::mutex g_scratch_mu;

// Device address of the fixed workspace on the current device.  In host code
// `g_scratch` only names a host-side stand-in, so the address is looked up
// once per device with that device current.
static int scratch_address(int device, void **out) {
  if (device < 0 || device >= 64) return fail(NKB_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(NKB_ERR_CUDA, std::string("cudaGetSymbolAddress(linear-attention scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[device] = ptr;
  }
  *out = g_scratch_addr[device];
  return NKB_OK;
}

}  // namespace linattn
}  // namespace nkb

extern "C" int nkb_linear_attention_noalloc(const void *q, const void *k, const void *v, void *out, int64_t B,
                                            int64_t H, int64_t T, int64_t D, void *stream) {
  using namespace nkb;
  using namespace nkb::linattn;
  if (!q || !k || !v || !out) return fail(NKB_ERR_INVALID, "linear attention: NULL pointer");
  if (D != linattn::D) return fail(NKB_ERR_UNSUPPORTED, "linear attention: head_dim must be 128");
  if (B < 0 || H < 0 || T < 0 || T % C) return fail(NKB_ERR_UNSUPPORTED, "linear attention: length must be a multiple of 64");
  if (B * H > INT32_MAX / 2 || T > INT32_MAX / 2) return fail(NKB_ERR_INVALID, "linear attention: sizes too large");
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  if (al & 15) return fail(NKB_ERR_UNSUPPORTED, "linear attention: pointers must be 16-byte aligned");
  if (B == 0 || H == 0 || T == 0) return NKB_OK;
  int dev = 0;
  NKB_CUDA_TRY(cudaGetDevice(&dev));
  const int BH = (int)(B * H);
  const int G = pick_segments(BH, (int)T, dev);
  const size_t need = G > 1 ? workspace_bytes(BH, G) : 0;
  if (need > (size_t)NKB_LINATTN_SCRATCH_BYTES)
    return fail(NKB_ERR_INVALID, "linear attention: " + std::to_string(B) + "x" + std::to_string(H) +
                                     " heads need " + std::to_string(need) + " bytes of workspace, more than the fixed " +
                                     std::to_string((size_t)NKB_LINATTN_SCRATCH_BYTES) + " bytes of the allocation-free entry point");
  void *ws = nullptr;
  if (int s = scratch_address(dev, &ws)) return s;
  Params p;
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.v = static_cast<const __nv_bfloat16 *>(v);
  p.o = static_cast<__nv_bfloat16 *>(out);
  p.ws = static_cast<float *>(ws);
  p.H = (int)H;
  p.BH = BH;
  p.T = (int)T;
  p.G = G;
  p.chunks_per_seg = G > 1 ? SEG_CHUNKS : (int)(T / C);
  const int64_t sb = H * T * D, sh = T * D, ss = D;
  p.qb = p.kb = p.vb = p.ob = sb;
  p.qh = p.kh = p.vh = p.oh = sh;
  p.qs = p.ks = p.vs = p.os = ss;
  return run(p, static_cast<cudaStream_t>(stream));
}
