// Attention of one new token against a resident KV cache (the decode step of
// the reference's Qwen3 loop: examples/models/qwen3/kernels/attention.py:
// 119-140 with start_pos, qwen3.py:310-336).  The traced composition is
//   scores = (q . k_s) * scale + mask[pos, s]     (mask: 0 for s <= pos, very
//   p = softmax(scores);  out = sum_s p_s v_s      negative above: a causal table)
// with q heads sharing KV heads (GQA: head h reads KV head h / n_rep).  Keys
// s > pos contribute nothing, so the kernel reads keys 0..pos only; pos comes
// from device memory (clamped into the cache as a gather index is).
//
// Split over keys ("flash-decoding"): CTA (b, g, c) takes KV head g of batch b,
// every query head of its group (their count a compile-time constant), and
// chunk c of the keys.  Four warps, each taking tiles of 32 keys: the warp
// issues the loads of its key rows (lane l: key base + l, 16 bytes at a time,
// all in flight) and of the first half of the tile's value rows (lane l
// owning features 4l..4l+3, coalesced, held in registers), scores every head
// of the group (q read from shared memory 16 bytes at a time), issues the
// second half of the value rows, folds the 32 scores into a running max / sum
// per head and accumulates sum_s p_s v_s from the registers.  The CTA writes its partial (max, sum, unnormalised output) per
// head; a second kernel merges the chunks of each (b, h).  fp32 throughout,
// bf16 output.
#include "common.cuh"

namespace nkb {
namespace decode {

constexpr int D = 128;          // head dimension
constexpr int MAX_REP = 8;      // query heads per KV head
constexpr int THREADS = 128;    // four warps
constexpr int KEY_TILE = 32;    // keys per warp step (one per lane)

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

__device__ __forceinline__ int64_t load_pos(const void *p, int dt) {
  const uint32_t raw = load_as_reg(p, 0, dt);
  return (dt == NKB_U32 || dt == NKB_U16 || dt == NKB_U8) ? (int64_t)raw : (int64_t)(int32_t)raw;
}

// R = query heads per KV head (compile-time: no work for absent heads).
template <int R>
__global__ void __launch_bounds__(THREADS, 2) attn_decode_kernel(const __grid_constant__ Params p) {
  __shared__ __align__(16) float s_q[R][D];
  __shared__ float s_m[4][R], s_l[4][R];
  __shared__ float s_o[4][R][D];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = blockIdx.x % p.splits, bg = blockIdx.x / p.splits;
  const int b = bg / p.HKV, g = bg % p.HKV;
  int64_t pos = load_pos(p.pos, p.pos_dt);
  pos = pos < 0 ? 0 : (pos >= p.S ? p.S - 1 : pos);
  const int len = (int)pos + 1;  // keys 0..pos
  const int k0 = c * p.chunk, k1 = min(k0 + p.chunk, len);

  for (int i = threadIdx.x; i < R * D; i += THREADS) {
    const int r = i / D, d = i % D;
    const int h = g * R + r;
    s_q[r][d] = __bfloat162float(p.q[(int64_t)b * p.qb + (int64_t)h * p.qh + d]) * p.scale;
  }
  __syncthreads();

  float m[R], l[R], o[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[r][j] = 0.f;
  }
  const __nv_bfloat16 *kbase = p.k + (int64_t)b * p.kb + (int64_t)g * p.kh;
  const __nv_bfloat16 *vbase = p.v + (int64_t)b * p.vb + (int64_t)g * p.vh;
  constexpr int HALF = KEY_TILE / 2;
#pragma unroll 1
  for (int t0 = k0 + warp * KEY_TILE; t0 < k1; t0 += 4 * KEY_TILE) {
    const int s = t0 + lane;
    const bool live = s < k1;
    const int nk = min(KEY_TILE, k1 - t0);
    // key row s (all 16-byte loads in flight) and the first half of the tile's
    // value rows (lane l: features 4l..4l+3; zeros past the chunk)
    uint4 kr[D / 8];
    const uint4 *krow = reinterpret_cast<const uint4 *>(kbase + (int64_t)(live ? s : t0) * p.ks);
#pragma unroll
    for (int j = 0; j < D / 8; ++j) kr[j] = krow[j];
    uint2 va[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j)
      va[j] = j < nk ? *reinterpret_cast<const uint2 *>(vbase + (int64_t)(t0 + j) * p.vs + 4 * lane) : make_uint2(0, 0);
    // scores of key s for every head of the group; q read 16 bytes at a time (broadcast)
    float sc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sc[r] = 0.f;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const __nv_bfloat162 *kk = reinterpret_cast<const __nv_bfloat162 *>(&kr[j]);
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(kk[e]);
        kf[2 * e] = f.x;
        kf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 qa = *reinterpret_cast<const float4 *>(&s_q[r][8 * j]);
        const float4 qb = *reinterpret_cast<const float4 *>(&s_q[r][8 * j + 4]);
        sc[r] = fmaf(qa.x, kf[0], sc[r]);
        sc[r] = fmaf(qa.y, kf[1], sc[r]);
        sc[r] = fmaf(qa.z, kf[2], sc[r]);
        sc[r] = fmaf(qa.w, kf[3], sc[r]);
        sc[r] = fmaf(qb.x, kf[4], sc[r]);
        sc[r] = fmaf(qb.y, kf[5], sc[r]);
        sc[r] = fmaf(qb.z, kf[6], sc[r]);
        sc[r] = fmaf(qb.w, kf[7], sc[r]);
      }
    }
    // second half of the value rows (the key registers are free now)
    uint2 vb[HALF];
#pragma unroll
    for (int j = 0; j < HALF; ++j)
      vb[j] = HALF + j < nk ? *reinterpret_cast<const uint2 *>(vbase + (int64_t)(t0 + HALF + j) * p.vs + 4 * lane)
                            : make_uint2(0, 0);
    // online softmax per head over the warp's 32 keys
    float pr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float x = live ? sc[r] : -INFINITY;
      float mx = x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[r], mx);      // finite: lane 0 of a tile is always live
      const float corr = __expf(m[r] - mn);  // 0 while m is -inf
      pr[r] = live ? __expf(x - mn) : 0.f;
      float sum = pr[r];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[r] = l[r] * corr + sum;
      m[r] = mn;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[r][j] *= corr;
    }
    // sum_s p_s v_s from the registers (p = 0 past the chunk)
#pragma unroll
    for (int j = 0; j < KEY_TILE; ++j) {
      const uint2 vv = j < HALF ? va[j] : vb[j - HALF];
      const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vv.x));
      const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vv.y));
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float pj = __shfl_sync(0xffffffffu, pr[r], j);
        o[r][0] = fmaf(pj, v01.x, o[r][0]);
        o[r][1] = fmaf(pj, v01.y, o[r][1]);
        o[r][2] = fmaf(pj, v23.x, o[r][2]);
        o[r][3] = fmaf(pj, v23.y, o[r][3]);
      }
    }
  }
  // merge the four warps' partials, then this chunk's partial per head -> workspace
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (lane == 0) {
      s_m[warp][r] = m[r];
      s_l[warp][r] = l[r];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_o[warp][r][4 * lane + j] = o[r][j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * D; i += THREADS) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][r]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float f = s_m[w][r] == -INFINITY ? 0.f : __expf(s_m[w][r] - M);
      L += s_l[w][r] * f;
      O += s_o[w][r][d] * f;
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

// out[b, h, :] = merge of the chunks' partials
__global__ void __launch_bounds__(D) attn_decode_combine_kernel(const __grid_constant__ Params p) {
  const int bh = blockIdx.x, d = threadIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const float *src = p.ws + (int64_t)bh * p.splits * (D + 2);
  float M = -INFINITY;
  for (int c = 0; c < p.splits; ++c) M = fmaxf(M, src[c * (D + 2)]);
  float L = 0.f, O = 0.f;
  for (int c = 0; c < p.splits; ++c) {
    const float mc = src[c * (D + 2)];
    const float f = mc == -INFINITY ? 0.f : __expf(mc - M);
    L += src[c * (D + 2) + 1] * f;
    O += src[c * (D + 2) + 2 + d] * f;
  }
  p.out[(int64_t)b * p.ob + (int64_t)h * p.oh + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

// The planner picks the chunk count (chunks of ~128 keys, at least four CTAs
// per SM in all) and sizes the workspace: B * H * splits * (D + 2) floats.
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
  switch (p.n_rep) {
    case 1: attn_decode_kernel<1><<<grid, THREADS, 0, a.stream>>>(p); break;
    case 2: attn_decode_kernel<2><<<grid, THREADS, 0, a.stream>>>(p); break;
    case 4: attn_decode_kernel<4><<<grid, THREADS, 0, a.stream>>>(p); break;
    case 8: attn_decode_kernel<8><<<grid, THREADS, 0, a.stream>>>(p); break;
    default: return fail(NKB_ERR_UNSUPPORTED, "attn_decode: 1, 2, 4 or 8 query heads per KV head");
  }
  if (int s = launch_status("attn_decode_kernel")) return s;
  attn_decode_combine_kernel<<<(unsigned)(p.B * p.H), D, 0, a.stream>>>(p);
  return launch_status("attn_decode_combine_kernel");
}

}  // namespace decode

NKB_REGISTER_KERNEL("attn_decode", decode::launch, decode::check);

}  // namespace nkb
