// Window matrix of a convolution (the reference's conv2d / conv3d, core/ops/conv.py:
// 230-312, lowered as one GEMM): cols[kk][m] with kk = (channel, kernel offset ...)
// and m = (batch, output position ...), read from the dense (B, C, *in) input,
// zero where a window reaches into the padding.  Replaces a pad launch and a
// strided copy: one read of the input (through L2) and one coalesced write of
// the matrix (contiguous along the innermost output axis).  Element size 2 or
// 4 bytes.
#include <algorithm>

#include <cstdlib>

#include "common.cuh"

namespace nkb {
namespace im2col {

constexpr int MAXN = 3;

struct Params {
  const void *x;
  void *cols;
  int n, esize;
  int64_t B, C, M, KK;
  int64_t in[MAXN], ks[MAXN], out[MAXN], stride[MAXN], pad[MAXN], dil[MAXN];
  int64_t in_plane;  // prod(in)
};

constexpr int RX = 64;   // threads along the innermost output axis
constexpr int RY = 4;    // output rows (batch, outer output axes) per block
constexpr int KKB = 16;  // window-matrix rows per block

// Block (rows r0..r0+3, kk0..kk0+15): thread (tx, ty) writes cols[kk][row * O + o]
// for o = tx, tx + 64, ...  The row is decomposed once; kk advances by carries.
template <typename T>
__global__ void __launch_bounds__(RX * RY) im2col_kernel(const __grid_constant__ Params p) {
  const T *x = static_cast<const T *>(p.x);
  T *cols = static_cast<T *>(p.cols);
  const int n = p.n;
  const int64_t O = p.out[n - 1];
  const int64_t rows = p.M / O;
  const int64_t row = (int64_t)blockIdx.x * RY + threadIdx.y;
  if (row >= rows) return;
  // row -> batch, outer output coordinates
  int64_t o_out[MAXN] = {0, 0, 0}, q = row;
  for (int d = n - 2; d >= 0; --d) {
    o_out[d] = q % p.out[d];
    q /= p.out[d];
  }
  const int64_t b = q;
  // first window row of the block -> channel, kernel offsets
  const int64_t kk0 = (int64_t)blockIdx.y * KKB;
  int64_t kof[MAXN] = {0, 0, 0}, r = kk0;
  for (int d = n - 1; d >= 0; --d) {
    kof[d] = r % p.ks[d];
    r /= p.ks[d];
  }
  int64_t c = r;
  const int64_t kk1 = min(p.KK, kk0 + KKB);
  for (int64_t kk = kk0; kk < kk1; ++kk) {
    // outer input coordinates of this row and window offset; valid or not
    int64_t base = (b * p.C + c) * p.in_plane, plane = 1;
    bool ok = true;
    for (int d = n - 2; d >= 0; --d) {
      plane *= p.in[d + 1];
      const int64_t i = o_out[d] * p.stride[d] + kof[d] * p.dil[d] - p.pad[d];
      ok = ok && i >= 0 && i < p.in[d];
      base += i * plane;
    }
    const int64_t s = p.stride[n - 1], shift = kof[n - 1] * p.dil[n - 1] - p.pad[n - 1], W = p.in[n - 1];
    T *dst = cols + kk * p.M + row * O;
    for (int64_t o = threadIdx.x; o < O; o += RX) {
      const int64_t i = o * s + shift;
      dst[o] = (ok && i >= 0 && i < W) ? x[base + i] : T(0);
    }
    // next window row: kernel offsets, then channel
    for (int d = n - 1; d >= 0; --d) {
      if (++kof[d] < p.ks[d]) break;
      kof[d] = 0;
      if (d == 0) ++c;
    }
  }
}

// Output rows of a multiple of 8 elements (bf16): thread g writes the 16-byte
// group of 8 consecutive elements g of each window row of its block (its
// output row decomposed once, the 8 inputs gathered from L1 / L2), so every
// store is 16 bytes and a warp writes 512 contiguous bytes.
constexpr int VT = 256;  // threads (groups of 8) per block
// I: the index type (32-bit when every index of the launch fits, fewer instructions)
template <typename I>
__global__ void __launch_bounds__(VT) im2col8_kernel(const __grid_constant__ Params p) {
  const uint16_t *x = static_cast<const uint16_t *>(p.x);
  uint16_t *cols = static_cast<uint16_t *>(p.cols);
  const int n = p.n;
  const I O = (I)p.out[n - 1], G = O / 8, M = (I)p.M;
  const I g = (I)blockIdx.x * VT + (I)threadIdx.x;  // group over (row, o / 8)
  if (g >= M / 8) return;
  const I row = g / G, o0 = (g - row * G) * 8;
  I ibase[MAXN] = {0, 0, 0}, q = row;  // window origin per outer input axis
  for (int d = n - 2; d >= 0; --d) {
    const I od = (I)p.out[d];
    const I o = q % od;
    q /= od;
    ibase[d] = o * (I)p.stride[d] - (I)p.pad[d];
  }
  const I b = q;
  const I kk0 = (I)blockIdx.y * KKB;
  I kof[MAXN] = {0, 0, 0}, r = kk0;
  for (int d = n - 1; d >= 0; --d) {
    kof[d] = r % (I)p.ks[d];
    r /= (I)p.ks[d];
  }
  I c = r;
  const I kk1 = min((I)p.KK, kk0 + KKB);
  const I s = (I)p.stride[n - 1], W = (I)p.in[n - 1], C = (I)p.C, plane_all = (I)p.in_plane;
  for (I kk = kk0; kk < kk1; ++kk) {
    I base = (b * C + c) * plane_all, plane = 1;
    bool ok = true;
    for (int d = n - 2; d >= 0; --d) {
      plane *= (I)p.in[d + 1];
      const I i = ibase[d] + kof[d] * (I)p.dil[d];
      ok = ok && i >= 0 && i < (I)p.in[d];
      base += i * plane;
    }
    const I i0 = o0 * s + kof[n - 1] * (I)p.dil[n - 1] - (I)p.pad[n - 1];
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const I ia = i0 + e * s, ib = ia + s;
      const uint32_t va = (ok && ia >= 0 && ia < W) ? x[base + ia] : 0u;
      const uint32_t vb = (ok && ib >= 0 && ib < W) ? x[base + ib] : 0u;
      w[e / 2] = va | (vb << 16);
    }
    *reinterpret_cast<uint4 *>(cols + (int64_t)kk * M + (int64_t)row * O + o0) = make_uint4(w[0], w[1], w[2], w[3]);
    for (int d = n - 1; d >= 0; --d) {
      if (++kof[d] < (I)p.ks[d]) break;
      kof[d] = 0;
      if (d == 0) ++c;
    }
  }
}

// 2-D 3x3 windows, stride 1, dilation 1, padding 1, bf16, rows of a multiple
// of 8 (the common "same" convolution): thread g owns 16-byte group g of every
// window row of its channel block.  For each (channel, kernel row) it loads the
// input chunk under its group and the two beside it (16-byte loads, mostly L1
// hits), and writes the three kernel columns as that chunk shifted by one
// element left, not at all, and right (funnel shifts): 3 loads and 3 stores per
// 24 outputs instead of 8 gathered elements per 8.
constexpr int CB3 = 2;  // channels per block (18 window rows)
__global__ void __launch_bounds__(VT) im2col3x3_kernel(const __grid_constant__ Params p) {
  const int G = (int)(p.in[1] / 8), H = (int)p.in[0], C = (int)p.C;
  const int M8 = (int)(p.M / 8);
  const int g = blockIdx.x * VT + threadIdx.x;  // group over (batch, output row, 8 columns)
  if (g >= M8) return;
  const int row = g / G, oc = g - row * G;
  const int b = row / H, oh = row - b * H;
  const uint4 *x4 = static_cast<const uint4 *>(p.x);
  uint4 *cols4 = static_cast<uint4 *>(p.cols);
  const int64_t M8l = M8;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  const int c0 = blockIdx.y * CB3, c1 = min(C, c0 + CB3);
  for (int c = c0; c < c1; ++c) {
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
      const int ih = oh + kh - 1;
      uint4 prev = zero, cur = zero, next = zero;
      if (ih >= 0 && ih < H) {
        const int64_t rb = (((int64_t)b * C + c) * H + ih) * G;  // 16-byte chunk index of the input row
        cur = x4[rb + oc];
        if (oc > 0) prev = x4[rb + oc - 1];
        if (oc + 1 < G) next = x4[rb + oc + 1];
      }
      // kernel column 0: input elements o - 1; 1: o; 2: o + 1
      const uint4 left = make_uint4(__funnelshift_l(prev.w, cur.x, 16), __funnelshift_l(cur.x, cur.y, 16),
                                    __funnelshift_l(cur.y, cur.z, 16), __funnelshift_l(cur.z, cur.w, 16));
      const uint4 right = make_uint4(__funnelshift_r(cur.x, cur.y, 16), __funnelshift_r(cur.y, cur.z, 16),
                                     __funnelshift_r(cur.z, cur.w, 16), __funnelshift_r(cur.w, next.x, 16));
      const int64_t kk = (int64_t)c * 9 + kh * 3;
      cols4[kk * M8l + g] = left;
      cols4[(kk + 1) * M8l + g] = cur;
      cols4[(kk + 2) * M8l + g] = right;
    }
  }
}

// "im2col": ptrs x cols; ints n esize B C in[n] ks[n] out[n] stride[n] pad_lo[n] dil[n]
int check(const Step &s) {
  if (s.buf_ids.size() != 2 || s.ints.size() < 4) return fail(NKB_ERR_PLAN, "im2col: bad parameters");
  const int64_t n = s.ints[0];
  if (n < 1 || n > MAXN || (int64_t)s.ints.size() != 4 + 6 * n) return fail(NKB_ERR_PLAN, "im2col: bad parameters");
  if (s.ints[1] != 2 && s.ints[1] != 4) return fail(NKB_ERR_UNSUPPORTED, "im2col: element size 2 or 4 bytes");
  for (int64_t i = 4; i < 4 + 6 * n; ++i)
    if (s.ints[i] < 0) return fail(NKB_ERR_PLAN, "im2col: negative size");
  return NKB_OK;
}

int launch(const LaunchArgs &a) {
  const auto &q = a.step->ints;
  Params p;
  p.x = a.ptrs[0];
  p.cols = a.ptrs[1];
  p.n = (int)q[0];
  p.esize = (int)q[1];
  p.B = q[2];
  p.C = q[3];
  p.in_plane = 1;
  int64_t kprod = 1, oprod = 1;
  for (int d = 0; d < p.n; ++d) {
    p.in[d] = q[4 + d];
    p.ks[d] = q[4 + p.n + d];
    p.out[d] = q[4 + 2 * p.n + d];
    p.stride[d] = q[4 + 3 * p.n + d];
    p.pad[d] = q[4 + 4 * p.n + d];
    p.dil[d] = q[4 + 5 * p.n + d];
    if (p.ks[d] < 1 || p.stride[d] < 1 || p.dil[d] < 1) return fail(NKB_ERR_PLAN, "im2col: bad window");
    p.in_plane *= p.in[d];
    kprod *= p.ks[d];
    oprod *= p.out[d];
  }
  p.M = p.B * oprod;
  p.KK = p.C * kprod;
  if (p.M == 0 || p.KK == 0) return NKB_OK;
  const int64_t rows = p.M / p.out[p.n - 1];
  const int64_t gy = (p.KK + KKB - 1) / KKB;
  const bool same3 = p.n == 2 && p.esize == 2 && p.ks[0] == 3 && p.ks[1] == 3 && p.stride[0] == 1 &&
                     p.stride[1] == 1 && p.dil[0] == 1 && p.dil[1] == 1 && p.pad[0] == 1 && p.pad[1] == 1 &&
                     p.out[0] == p.in[0] && p.out[1] == p.in[1] && p.in[1] % 8 == 0;
  if (same3 && ((reinterpret_cast<uintptr_t>(p.cols) | reinterpret_cast<uintptr_t>(p.x)) & 15) == 0 &&
      p.M / 8 <= INT32_MAX / 2 && p.B * p.C * p.in_plane / 8 <= INT32_MAX / 2 && (p.C + CB3 - 1) / CB3 <= 65535 &&
      !getenv("NKB_IM2COL_INDEX64")) {
    dim3 grid((unsigned)((p.M / 8 + VT - 1) / VT), (unsigned)((p.C + CB3 - 1) / CB3));
    im2col3x3_kernel<<<grid, VT, 0, a.stream>>>(p);
    return launch_status("im2col3x3_kernel");
  }
  if (p.esize == 2 && p.out[p.n - 1] % 8 == 0 && (reinterpret_cast<uintptr_t>(p.cols) & 15) == 0 &&
      gy <= 65535 && (p.M / 8 + VT - 1) / VT <= INT32_MAX) {
    dim3 grid((unsigned)((p.M / 8 + VT - 1) / VT), (unsigned)gy);
    // 32-bit indices when the input, the matrix row length and every window coordinate fit
    int64_t lim = std::max<int64_t>(p.B * p.C * p.in_plane, p.M + VT * 8);
    for (int d = 0; d < p.n; ++d)
      lim = std::max<int64_t>(lim, (p.out[d] + 8) * p.stride[d] + p.ks[d] * p.dil[d] + p.pad[d] + p.in[d]);
    // NKB_IM2COL_INDEX64 (any value) takes the 64-bit instantiation at any size:
    // the switch the tests use to run it on small inputs
    if (lim < INT32_MAX / 2 && !getenv("NKB_IM2COL_INDEX64"))
      im2col8_kernel<int32_t><<<grid, VT, 0, a.stream>>>(p);
    else
      im2col8_kernel<int64_t><<<grid, VT, 0, a.stream>>>(p);
    return launch_status("im2col8_kernel");
  }
  if (gy > 65535 || (rows + RY - 1) / RY > INT32_MAX) return fail(NKB_ERR_UNSUPPORTED, "im2col: too large");
  dim3 grid((unsigned)((rows + RY - 1) / RY), (unsigned)gy);
  dim3 block(RX, RY);
  if (p.esize == 2)
    im2col_kernel<uint16_t><<<grid, block, 0, a.stream>>>(p);
  else
    im2col_kernel<uint32_t><<<grid, block, 0, a.stream>>>(p);
  return launch_status("im2col_kernel");
}

}  // namespace im2col

NKB_REGISTER_KERNEL("im2col", im2col::launch, im2col::check);

}  // namespace nkb
