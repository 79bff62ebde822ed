// Attention of one new token against a resident KV cache (the decode step of
// the reference's Qwen3 loop: examples/models/qwen3/kernels/attention.py:
// 119-140 with start_pos, qwen3.py:310-336).  The traced composition is
//   scores = (q . k_s) * scale + mask[pos, s]     (mask: 0 for s <= pos, very
//   p = softmax(scores);  out = sum_s p_s v_s      negative above: a causal table)
// with q heads sharing KV heads (GQA: head h reads KV head h / n_rep).  Keys
// s > pos contribute nothing, so the kernel reads keys 0..pos only; pos comes
// from device memory (clamped into the cache as a gather index is).
//
// Split over keys ("flash-decoding"): CTA (b, g, c) takes KV head g of batch b
// and chunk c of the keys.  The R query heads of the group form the rows of
// one m16 tensor-core tile (rows >= R zero), so scores and PV run on bf16
// mma.sync m16n8k16 with fp32 accumulation: per 16-key tile S = Q K^T (16 mma)
// and O += P V (16 mma), P converted to bf16 in registers.  Four warps per
// CTA, each taking every fourth tile of the chunk through its own
// double-buffered, XOR-swizzled shared-memory ring filled by cp.async.  The
// CTA writes its partial (max, sum, unnormalised output) per head; a second
// kernel merges the chunks of each (b, h).  fp32 softmax, bf16 output.
#include "common.cuh"
#include "mma_sync.cuh"

namespace nkb {
namespace decode {

constexpr int D = 128;          // head dimension
constexpr int MAX_REP = 8;      // query heads per KV head
constexpr int THREADS = 128;    // four warps

struct Params {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16 *out;
  const void *pos;
  int pos_dt;
  int B, H, HKV, S, n_rep, chunk, splits;
  int64_t qb, qh, kb, kh, ks, vb, vh, vs, ob, oh;  // element strides (feature stride 1)
  float scale;
  float *ws;  // [B][H][splits][D + 2]: max, sum, output
};

// out[b, h, d] from the chunks' partials (max, sum, unnormalised output)
__device__ __forceinline__ void merge_head(const Params &p, int b, int h, int d) {
  const float *src = p.ws + ((int64_t)b * p.H + h) * p.splits * (D + 2);
  float M = -INFINITY;
#pragma unroll 4  // the splits' loads in flight together
  for (int c = 0; c < p.splits; ++c) M = fmaxf(M, __ldcg(src + c * (D + 2)));
  float L = 0.f, O = 0.f;
#pragma unroll 4
  for (int c = 0; c < p.splits; ++c) {
    const float mc = __ldcg(src + c * (D + 2));
    const float f = mc == -INFINITY ? 0.f : __expf(mc - M);
    L += __ldcg(src + c * (D + 2) + 1) * f;
    O += __ldcg(src + c * (D + 2) + 2 + d) * f;
  }
  p.out[(int64_t)b * p.ob + (int64_t)h * p.oh + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

__device__ __forceinline__ int64_t load_pos(const void *p, int dt) {
  const uint32_t raw = load_as_reg(p, 0, dt);
  return (dt == NKB_U32 || dt == NKB_U16 || dt == NKB_U8) ? (int64_t)raw : (int64_t)(int32_t)raw;
}

using namespace mma;
// byte offset of 16-byte chunk `chunk` of row `row` in a swizzled [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return mma::swz(row, chunk, D * 2); }

constexpr int BN = 16;                      // keys per tile
constexpr int TILE_BYTES = BN * D * 2;      // 4 KB per K or V tile
constexpr int WARP_SMEM = 2 * 2 * TILE_BYTES;  // two stages of K and V per warp

// CTA (b, g, c): the R query heads of KV head g form the rows of one m16 tile
// (rows >= R are zero).  Each warp takes every fourth 16-key tile of chunk c,
// double-buffered in its own swizzled shared-memory ring by cp.async, and
// runs S = Q K^T (16 mma), an online softmax on the score fragments, and
// O += P V (16 mma) with P converted to bf16 in registers.
template <int R>
__global__ void __launch_bounds__(THREADS, 2) attn_decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *sQ = smem;                                   // 16 rows x 128, swizzled
  uint8_t *sRing = smem + 16 * D * 2;                   // 4 warps x WARP_SMEM
  float *s_o = reinterpret_cast<float *>(sRing + 4 * WARP_SMEM);  // [4][R][D]
  float *s_m = s_o + 4 * R * D;                         // [4][R]
  float *s_l = s_m + 4 * R;                             // [4][R]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = blockIdx.x % p.splits, bg = blockIdx.x / p.splits;
  const int b = bg / p.HKV, g = bg % p.HKV;
  pdl_wait();
  pdl_trigger();
  int64_t pos = load_pos(p.pos, p.pos_dt);
  pos = pos < 0 ? 0 : (pos >= p.S ? p.S - 1 : pos);
  const int len = (int)pos + 1;  // keys 0..pos
  const int k0 = c * p.chunk, k1 = min(k0 + p.chunk, len);
  const __nv_bfloat16 *kbase = p.k + (int64_t)b * p.kb + (int64_t)g * p.kh;
  const __nv_bfloat16 *vbase = p.v + (int64_t)b * p.vb + (int64_t)g * p.vh;

  // Q rows (zero past R): 16 rows x 16 chunks of 16 bytes
  for (int i = threadIdx.x; i < 16 * (D / 8); i += THREADS) {
    const int r = i / (D / 8), ch = i % (D / 8);
    const bool ok = r < R;
    const __nv_bfloat16 *src = p.q + (int64_t)b * p.qb + (int64_t)(g * R + (ok ? r : 0)) * p.qh + ch * 8;
    cp_async16(smem_addr(sQ) + swz(r, ch), src, ok);
  }
  cp_commit();

  // this warp's tiles: ts = k0 + (warp + 4 i) * BN, while ts < k1
  const int n_tiles = k1 > k0 ? (k1 - k0 + BN - 1) / BN : 0;
  const int my_tiles = n_tiles > warp ? (n_tiles - warp + 3) / 4 : 0;
  uint8_t *ring = sRing + warp * WARP_SMEM;
  auto load_tile = [&](int i, int stage) {
    const int ts = k0 + (warp + 4 * i) * BN;
    const uint32_t kd = smem_addr(ring + stage * 2 * TILE_BYTES), vd = kd + TILE_BYTES;
#pragma unroll
    for (int j = 0; j < BN * (D / 8) / 32; ++j) {  // 8 chunks of K and 8 of V per lane
      const int idx = j * 32 + lane, r = idx / (D / 8), ch = idx % (D / 8);
      const int key = ts + r;
      const bool ok = key < k1;
      const int64_t kr = ok ? key : k0;
      cp_async16(kd + swz(r, ch), kbase + kr * p.ks + ch * 8, ok);
      cp_async16(vd + swz(r, ch), vbase + kr * p.vs + ch * 8, ok);
    }
  };
  if (my_tiles > 0) load_tile(0, 0);
  cp_commit();

  // Q fragments (A operand, rows = heads), kept in registers
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk)
    ldsm_x4(smem_addr(sQ) + swz(lane % 16, kk * 2 + lane / 16), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

#pragma unroll 1
  for (int i = 0; i < my_tiles; ++i) {
    const int stage = i & 1;
    __syncwarp();  // every lane is done reading the stage the next load overwrites
    if (i + 1 < my_tiles) load_tile(i + 1, stage ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncwarp();  // this tile's copies, issued by every lane, are visible
    const uint32_t kt = smem_addr(ring + stage * 2 * TILE_BYTES), vt = kt + TILE_BYTES;
    const int ts = k0 + (warp + 4 * i) * BN;
    // S = Q K^T: 16 rows (heads) x 16 keys
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t b0, b1, b2, b3;
      const int r = (lane % 8) + (lane / 16) * 8;
      ldsm_x4(kt + swz(r, kk * 2 + (lane / 8) % 2), b0, b1, b2, b3);
      mma16816(s[0], qf[kk], b0, b1);
      mma16816(s[1], qf[kk], b2, b3);
    }
    // scale, mask keys past the chunk / the position, online softmax per row
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = ts + j * 8 + (lane % 4) * 2 + (e & 1);
        const float v = key < k1 ? s[j][e] * p.scale : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int r2 = 0; r2 < 2; ++r2) {
      mx[r2] = fmaxf(mx[r2], __shfl_xor_sync(0xffffffffu, mx[r2], 1));
      mx[r2] = fmaxf(mx[r2], __shfl_xor_sync(0xffffffffu, mx[r2], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r2 = 0; r2 < 2; ++r2) {
      alpha[r2] = __expf(m_r[r2] - mx[r2]);  // 0 while m was -inf (the first key of a tile is in range)
      m_r[r2] = mx[r2];
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = __expf(s[j][e] - m_r[e >> 1]);
        s[j][e] = pv;
        rs[e >> 1] += pv;
      }
    uint32_t pf[4];
    pf[0] = pack2(s[0][0], s[0][1]);
    pf[1] = pack2(s[0][2], s[0][3]);
    pf[2] = pack2(s[1][0], s[1][1]);
    pf[3] = pack2(s[1][2], s[1][3]);
#pragma unroll
    for (int r2 = 0; r2 < 2; ++r2) l_r[r2] = l_r[r2] * alpha[r2] + rs[r2];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // O += P V: V tile read transposed by ldmatrix
#pragma unroll
    for (int j = 0; j < D / 8; j += 2) {
      uint32_t b0, b1, b2, b3;
      const int r = (lane % 8) + ((lane / 8) % 2) * 8;
      ldsm_x4_t(vt + swz(r, j + lane / 16), b0, b1, b2, b3);
      mma16816(o[j], pf, b0, b1);
      mma16816(o[j + 1], pf, b2, b3);
    }
  }
  // row sums across the quad; rows (heads) < R go to the merge buffers
#pragma unroll
  for (int r2 = 0; r2 < 2; ++r2) {
    l_r[r2] += __shfl_xor_sync(0xffffffffu, l_r[r2], 1);
    l_r[r2] += __shfl_xor_sync(0xffffffffu, l_r[r2], 2);
  }
#pragma unroll
  for (int r2 = 0; r2 < 2; ++r2) {
    const int row = lane / 4 + r2 * 8;
    if (row < R) {
      if (lane % 4 == 0) {
        s_m[warp * R + row] = m_r[r2];
        s_l[warp * R + row] = l_r[r2];
      }
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        const int col = j * 8 + (lane % 4) * 2;
        s_o[(warp * R + row) * D + col] = o[j][2 * r2];
        s_o[(warp * R + row) * D + col + 1] = o[j][2 * r2 + 1];
      }
    }
  }
  __syncthreads();
  // this chunk's partial per head (max, sum, unnormalised output) -> workspace
  for (int i = threadIdx.x; i < R * D; i += THREADS) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w * R + r]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = s_m[w * R + r];
      const float f = mw == -INFINITY ? 0.f : __expf(mw - M);
      L += s_l[w * R + r] * f;
      O += s_o[(w * R + r) * D + d] * f;
    }
    const int h = g * R + r;
    float *dst = p.ws + (((int64_t)b * p.H + h) * p.splits + c) * (D + 2);
    if (d == 0) {
      dst[0] = M;
      dst[1] = L;
    }
    dst[2 + d] = O;
  }
}

template <int R>
constexpr int smem_bytes() {
  return 16 * D * 2 + 4 * WARP_SMEM + (4 * R * D + 8 * R) * 4;
}

// out[b, h, :] = merge of the chunks' partials
__global__ void __launch_bounds__(D) attn_decode_combine_kernel(const __grid_constant__ Params p) {
  const int bh = blockIdx.x, d = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  merge_head(p, bh / p.H, bh % p.H, d);
}

// The planner picks the chunk count (chunks of ~512 keys, at least one CTA per
// SM in all) and sizes the workspace: B * H * splits * (D + 2) floats.
// "attn_decode": ptrs q k v out pos ws; ints B H HKV S D splits pos_dtype
//                qb qh kb kh ks vb vh vs ob oh; floats scale
int check(const Step &s) {
  if (s.buf_ids.size() != 6 || s.ints.size() != 17 || s.floats.size() != 1)
    return fail(NKB_ERR_PLAN, "attn_decode: bad parameters");
  const auto &q = s.ints;
  if (q[4] != D) return fail(NKB_ERR_UNSUPPORTED, "attn_decode: head_dim must be 128");
  if (q[2] <= 0 || q[1] % q[2] || q[1] / q[2] > MAX_REP || ((q[1] / q[2]) & (q[1] / q[2] - 1)))
    return fail(NKB_ERR_UNSUPPORTED, "attn_decode: 1, 2, 4 or 8 query heads per KV head");
  if (q[5] < 1 || q[0] < 0 || q[3] < 1) return fail(NKB_ERR_PLAN, "attn_decode: sizes out of range");
  for (int i = 7; i < 17; ++i)
    if (q[i] < 0 || q[i] % 8) return fail(NKB_ERR_UNSUPPORTED, "attn_decode: strides must be multiples of 8");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  for (int i = 0; i < 4; ++i)
    if (reinterpret_cast<uintptr_t>(a.ptrs[i]) & 15) return fail(NKB_ERR_UNSUPPORTED, "attn_decode: unaligned operand");
  Params p;
  p.q = static_cast<const __nv_bfloat16 *>(a.ptrs[0]);
  p.k = static_cast<const __nv_bfloat16 *>(a.ptrs[1]);
  p.v = static_cast<const __nv_bfloat16 *>(a.ptrs[2]);
  p.out = static_cast<__nv_bfloat16 *>(a.ptrs[3]);
  p.pos = a.ptrs[4];
  p.ws = static_cast<float *>(a.ptrs[5]);
  p.B = (int)q[0];
  p.H = (int)q[1];
  p.HKV = (int)q[2];
  p.S = (int)q[3];
  p.splits = (int)q[5];
  p.pos_dt = (int)q[6];
  p.qb = q[7];
  p.qh = q[8];
  p.kb = q[9];
  p.kh = q[10];
  p.ks = q[11];
  p.vb = q[12];
  p.vh = q[13];
  p.vs = q[14];
  p.ob = q[15];
  p.oh = q[16];
  p.n_rep = p.H / p.HKV;
  p.chunk = (p.S + p.splits - 1) / p.splits;
  p.scale = a.step->floats[0];
  if (p.B == 0) return NKB_OK;
  const unsigned grid = (unsigned)(p.B * p.HKV * p.splits);
  static ContextOnce attr_set[4];
  auto go = [&](auto kern, int smem, int slot) -> int {
    if (int s = attr_set[slot].run(a.device, [&]() -> int {
          NKB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
          return NKB_OK;
        }))
      return s;
    NKB_CUDA_TRY(launch_pdl(a.pdl, kern, grid, THREADS, smem, a.stream, p));
    return NKB_OK;
  };
  int st = NKB_OK;
  switch (p.n_rep) {
    case 1: st = go(attn_decode_kernel<1>, smem_bytes<1>(), 0); break;
    case 2: st = go(attn_decode_kernel<2>, smem_bytes<2>(), 1); break;
    case 4: st = go(attn_decode_kernel<4>, smem_bytes<4>(), 2); break;
    case 8: st = go(attn_decode_kernel<8>, smem_bytes<8>(), 3); break;
    default: return fail(NKB_ERR_UNSUPPORTED, "attn_decode: 1, 2, 4 or 8 query heads per KV head");
  }
  if (st) return st;
  if (int s = launch_status("attn_decode_kernel")) return s;
  launch_pdl(true, attn_decode_combine_kernel, (unsigned)(p.B * p.H), D, 0, a.stream, p);
  return launch_status("attn_decode_combine_kernel");
}

}  // namespace decode

NKB_REGISTER_KERNEL("attn_decode", decode::launch, decode::check);

}  // namespace nkb
