// Producer side of the video self-attention (SelfAttention.forward,
// hymm/models/modules/wan_video_dit.py:699-705, 764-787): after the q / k / v
// projections, RMSNorm of q and k over the full hidden width (torch.nn.RMSNorm,
// :226-227), 3D RoPE of q and k in float64 complex arithmetic (rope_apply_head_dim,
// :177-182) and the Ulysses all-to-all pack (all_to_all_4D's send layout
// [P, S/P, H/P, D], head padding to P * hp heads, :775-787), fused into one pass
// per token row; and its backward.
//
// Numerics follow the reference's op sequence: the norm in fp32
// (x * rsqrt(mean(x^2) + eps)) * gamma rounded to bf16; the rotation of that bf16
// pair, (a c - b s, a s + b c), which the reference evaluates in double and rounds
// to float, then to bf16 (its double -> bf16 conversion goes through float).  Here
// the rotation is evaluated in float-float arithmetic from a table of cos / sin
// split into float hi + lo parts (rope_ff [S][D/2][4] = cos_hi, cos_lo, sin_hi,
// sin_lo): a * c_hi is exact as a two-product (a bf16 has 8 significant bits),
// a * c_lo lies below the float rounding level, and the two products are added with
// a two-sum, so the float result is the correctly rounded value of the exact
// rotation except within ~2^-46 of a float rounding midpoint, where the reference's
// double path may round differently (then the bf16 results still agree unless that
// float lies on a bf16 midpoint).  Backward: the conjugate rotation the same way,
// rounded to bf16, then the RMSNorm gradient in fp32.  Built with -fmad=false (every
// product and sum rounds once; the two-products are explicit fmaf).
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "prism_bsa.h"
#include "prism_common.cuh"

namespace prism {

constexpr int kProdThreads = 128;

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}
__device__ __forceinline__ float f2bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// a c + b s (sign = +1) or a c - b s (sign = -1) with a, b bf16 values, c = c_hi + c_lo,
// s = s_hi + s_lo: two-products of the hi parts, lo parts folded into the error
// terms, a two-sum of the products, rounded once to float.
__device__ __forceinline__ float ff_dot2(float a, float chi, float clo, float b, float shi, float slo,
                                         float sign) {
  const float p1 = __fmul_rn(a, chi);
  const float e1 = __fmaf_rn(a, clo, __fmaf_rn(a, chi, -p1));
  const float bs = sign * b;
  const float p2 = __fmul_rn(bs, shi);
  const float e2 = __fmaf_rn(bs, slo, __fmaf_rn(bs, shi, -p2));
  const float sum = __fadd_rn(p1, p2);
  const float bb = __fsub_rn(sum, p1);
  const float err = __fadd_rn(__fsub_rn(p1, __fsub_rn(sum, bb)), __fsub_rn(p2, bb));
  return __fadd_rn(sum, __fadd_rn(err, __fadd_rn(e1, e2)));
}

__device__ float block_sum_f(float v, float* red) {
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s = __fadd_rn(s, red[i]);
  return s;
}

// One CTA per packed row s < S_pack.  x rows [S, C] (C = H * D, row stride ld
// elements); out [P][S_pack][hp][D] with P * hp >= H (heads h >= H are zero, rows
// s >= S are zero: the last rank's padding of an uneven split).  norm = 0: v
// (copy); norm = 1: RMSNorm + RoPE with rope_ff [S][D/2] float4 (cos_hi, cos_lo,
// sin_hi, sin_lo).  A
// thread holds its kV 8-column groups of the row in registers between the norm's
// reduction and the rotation (kV = ceil(C / 8 / kProdThreads)).
template <int kV>
__global__ void __launch_bounds__(kProdThreads) norm_rope_pack_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t S, int64_t S_pack, int H, int D, int P,
    int hp, const float* __restrict__ gamma, float eps, const float4* __restrict__ rope_ff, int norm,
    __nv_bfloat16* __restrict__ out, float* __restrict__ rstd_out) {
  extern __shared__ float4 cs[];  // D/2 rotations of this token
  __shared__ float red[32];
  const int64_t s = blockIdx.x;
  if (s >= S) {  // padding row (uniform per CTA)
    for (int i = threadIdx.x; i < P * hp * D / 8; i += blockDim.x) {
      const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
      reinterpret_cast<uint4*>(out + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int C = H * D;
  const uint4* xr = reinterpret_cast<const uint4*>(x + s * ld);
  const int nv = C / 8;
  uint4 xv[kV];
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i = threadIdx.x + k * kProdThreads;
    xv[k] = i < nv ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
  }
  float r = 1.0f;
  if (norm) {
    for (int i = threadIdx.x; i < D / 2; i += blockDim.x) cs[i] = __ldg(rope_ff + s * (D / 2) + i);
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const uint32_t u[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf_lo(u[j]), b = bf_hi(u[j]);
        ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
      }
    }
    const float tot = block_sum_f(ss, red);
    r = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)C), eps));
    if (threadIdx.x == 0) rstd_out[s] = r;
    __syncthreads();  // cs visible
  }
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i = threadIdx.x + k * kProdThreads;
    if (i >= nv) break;
    const int col = i * 8;
    const int h = col / D, d0 = col - h * D;
    uint4 o = xv[k];
    if (norm) {
      const uint32_t u[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      uint32_t w[4];
      const float4 g0 = gamma ? reinterpret_cast<const float4*>(gamma + col)[0] : make_float4(1, 1, 1, 1);
      const float4 g1 = gamma ? reinterpret_cast<const float4*>(gamma + col)[1] : make_float4(1, 1, 1, 1);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // normed pair, rounded to bf16 (the RMSNorm output dtype)
        const float a = f2bf(__fmul_rn(__fmul_rn(bf_lo(u[j]), r), g[2 * j]));
        const float b = f2bf(__fmul_rn(__fmul_rn(bf_hi(u[j]), r), g[2 * j + 1]));
        const float4 t = cs[(d0 >> 1) + j];  // cos_hi, cos_lo, sin_hi, sin_lo
        w[j] = pack2(ff_dot2(a, t.x, t.y, b, t.z, t.w, -1.0f), ff_dot2(a, t.z, t.w, b, t.x, t.y, 1.0f));
      }
      o = make_uint4(w[0], w[1], w[2], w[3]);
    }
    const int p = h / hp, hh = h - p * hp;
    reinterpret_cast<uint4*>(out + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0] = o;
  }
  // padded heads of the packed row
  for (int i = nv + threadIdx.x; i < P * hp * D / 8; i += blockDim.x) {
    const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
    reinterpret_cast<uint4*>(out + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0] = make_uint4(0, 0, 0, 0);
  }
}

// Backward.  g [P][S_pack][hp][D]: gradient of the packed output.  With
// dy = the conjugate rotation of g (float-float, rounded to bf16) and
// r = rstd[s]:
//   dx = r (gamma dy) - x r^3 / C * dot,  dot = sum over the row of gamma dy x,
//   dgamma = sum over rows of dy x r.
// Phase A: one warp per row computes dot.  Phase B: one thread per 8 columns of a
// 32-row tile writes dx and its tile's dgamma partial [S / 32][C]; norm = 0 is the
// unpack alone.
__device__ __forceinline__ void rot_back8(const uint4 gv, const float4* __restrict__ ffrow, int d0,
                                          float dy[8]) {
  const uint32_t gu[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 t = __ldg(ffrow + (d0 >> 1) + j);  // cos_hi, cos_lo, sin_hi, sin_lo
    const float ga = bf_lo(gu[j]), gb = bf_hi(gu[j]);
    // gradient through (a + ib)(c + is): the conjugate rotation
    dy[2 * j] = f2bf(ff_dot2(ga, t.x, t.y, gb, t.z, t.w, 1.0f));
    dy[2 * j + 1] = f2bf(ff_dot2(gb, t.x, t.y, ga, t.z, t.w, -1.0f));
  }
}

__global__ void norm_rope_dot_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                     int64_t ld, int64_t S, int64_t S_pack, int H, int D, int hp,
                                     const float* __restrict__ gamma, const float4* __restrict__ rope_ff,
                                     float* __restrict__ dot) {
  const int64_t s = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (s >= S) return;
  const int nv = H * D / 8;
  const float4* csrow = rope_ff + s * (D / 2);
  float acc = 0.0f;
#pragma unroll 4
  for (int i = lane; i < nv; i += 32) {
    const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g + (((int64_t)p * S_pack + s) * hp + hh) * D + d0));
    const uint4 xq = __ldg(reinterpret_cast<const uint4*>(x + s * ld) + i);
    float gm[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
    if (gamma) {
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + col));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + col) + 1);
      gm[0] = g0.x; gm[1] = g0.y; gm[2] = g0.z; gm[3] = g0.w;
      gm[4] = g1.x; gm[5] = g1.y; gm[6] = g1.z; gm[7] = g1.w;
    }
    float dy[8];
    rot_back8(gv, csrow, d0, dy);
    const uint32_t xu[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float xj = (j & 1) ? bf_hi(xu[j >> 1]) : bf_lo(xu[j >> 1]);
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(gm[j], dy[j]), xj));
    }
  }
  for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if (lane == 0) dot[s] = acc;
}

constexpr int kProdTileRows = 32;
__global__ void __launch_bounds__(kProdThreads) norm_rope_dx_kernel(
    const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t S,
    int64_t S_pack, int H, int D, int hp, const float* __restrict__ gamma, const float* __restrict__ rstd,
    const float* __restrict__ dot, const float4* __restrict__ rope_ff, int norm,
    __nv_bfloat16* __restrict__ dx, int64_t ldx, float* __restrict__ dgamma_part) {
  const int C = H * D, nv = C / 8;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // 8-column group
  if (i >= nv) return;
  const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
  const int64_t s0 = (int64_t)blockIdx.y * kProdTileRows;
  float gm[8], dg[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    gm[j] = (norm && gamma) ? __ldg(gamma + col + j) : 1.0f;
    dg[j] = 0.0f;
  }
#pragma unroll 2
  for (int rr = 0; rr < kProdTileRows; ++rr) {
    const int64_t s = s0 + rr;
    if (s >= S) break;
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g + (((int64_t)p * S_pack + s) * hp + hh) * D + d0));
    uint4* dst = reinterpret_cast<uint4*>(dx + s * ldx + col);
    if (!norm) {
      *dst = gv;
      continue;
    }
    const uint4 xq = __ldg(reinterpret_cast<const uint4*>(x + s * ld) + i);
    float dy[8];
    rot_back8(gv, rope_ff + s * (D / 2), d0, dy);
    const float r = __ldg(rstd + s);
    const float coef = __fdiv_rn(__fmul_rn(__fmul_rn(__fmul_rn(r, r), r), __ldg(dot + s)), (float)C);
    const uint32_t xu[4] = {xq.x, xq.y, xq.z, xq.w};
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float o[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int jj = 2 * j + e;
        const float xj = e ? bf_hi(xu[j]) : bf_lo(xu[j]);
        o[e] = __fsub_rn(__fmul_rn(r, __fmul_rn(gm[jj], dy[jj])), __fmul_rn(xj, coef));
        dg[jj] = __fadd_rn(dg[jj], __fmul_rn(dy[jj], __fmul_rn(xj, r)));
      }
      w[j] = pack2(o[0], o[1]);
    }
    *dst = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (norm && dgamma_part != nullptr) {
    float4* dp = reinterpret_cast<float4*>(dgamma_part + (int64_t)blockIdx.y * C + col);
    dp[0] = make_float4(dg[0], dg[1], dg[2], dg[3]);
    dp[1] = make_float4(dg[4], dg[5], dg[6], dg[7]);
  }
}

// out[y][c] = sum over rows b in [y * per, y * per + per) of part[b][c] (sequential in
// b), one thread per column; blockIdx.y = row group.
__global__ void column_sum_kernel(const float* __restrict__ part, int64_t rows, int64_t per, int C,
                                  float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int64_t b0 = (int64_t)blockIdx.y * per, b1 = b0 + per < rows ? b0 + per : rows;
  float s = 0.0f;
#pragma unroll 8
  for (int64_t b = b0; b < b1; ++b) s = __fadd_rn(s, __ldg(part + b * C + c));
  out[(int64_t)blockIdx.y * C + c] = s;
}

}  // namespace prism

using namespace prism;

extern "C" {

prism_status_t prism_norm_rope_pack(const void* x, int64_t ld, int64_t S, int64_t S_pack, int H, int D,
                                    int P, int hp, const float* gamma, float eps, const float* rope_ff,
                                    int norm, void* out, float* rstd, cudaStream_t stream) {
  PRISM_CHECK_ARG(x && out && (!norm || (rope_ff && rstd)), "prism_norm_rope_pack: null pointer");
  PRISM_CHECK_ARG(S >= 0 && S_pack >= S && S_pack < (int64_t)1 << 31 && H >= 1 && D >= 8 && D % 8 == 0 &&
                      P >= 1 && hp >= 1 && P * hp >= H && ld % 8 == 0 && ld >= (int64_t)H * D &&
                      (int64_t)H * D <= 8 * 8 * kProdThreads,
                  "prism_norm_rope_pack: bad sizes (hidden width <= %d)", 8 * 8 * kProdThreads);
  PRISM_CHECK_ARG(aligned16(x) && aligned16(out) && (gamma == nullptr || aligned16(gamma)) &&
                      (rope_ff == nullptr || aligned16(rope_ff)),
                  "prism_norm_rope_pack: tensors must be 16-byte aligned");
  if (S_pack == 0) return PRISM_OK;
  const int nvt = (H * D / 8 + kProdThreads - 1) / kProdThreads;
  const size_t sm = norm ? (D / 2) * sizeof(float4) : 0;
#define PRISM_NRP_FWD(V)                                                                              \
  norm_rope_pack_kernel<V><<<(unsigned)S_pack, kProdThreads, sm, stream>>>(                           \
      (const __nv_bfloat16*)x, ld, S, S_pack, H, D, P, hp, gamma, eps, (const float4*)rope_ff, norm,       \
      (__nv_bfloat16*)out,                                                                             \
      rstd)
  switch (nvt) {
    case 1: PRISM_NRP_FWD(1); break;
    case 2: PRISM_NRP_FWD(2); break;
    case 3: PRISM_NRP_FWD(3); break;
    case 4: PRISM_NRP_FWD(4); break;
    case 5: PRISM_NRP_FWD(5); break;
    case 6: PRISM_NRP_FWD(6); break;
    case 7: PRISM_NRP_FWD(7); break;
    default: PRISM_NRP_FWD(8); break;
  }
#undef PRISM_NRP_FWD
  PRISM_CHECK_LAUNCH("prism_norm_rope_pack");
  return PRISM_OK;
}

size_t prism_norm_rope_pack_bwd_workspace_bytes(int64_t S, int H, int D) {
  const size_t tiles = (size_t)((S + kProdTileRows - 1) / kProdTileRows);
  // dot [S], dgamma partials [tiles][C], second-level partials [<= 64][C]
  return ((size_t)S + (tiles + 64) * (size_t)H * D) * sizeof(float) + 256;
}

prism_status_t prism_norm_rope_pack_bwd(const void* g, const void* x, int64_t ld, int64_t S, int64_t S_pack,
                                        int H, int D, int P, int hp, const float* gamma, const float* rstd,
                                        const float* rope_ff, int norm, void* dx, int64_t ldx,
                                        void* workspace, float* dgamma, cudaStream_t stream) {
  PRISM_CHECK_ARG(g && dx && (!norm || (x && rstd && rope_ff && workspace && dgamma)),
                  "prism_norm_rope_pack_bwd: null pointer");
  PRISM_CHECK_ARG(S >= 0 && S_pack >= S && S < (int64_t)1 << 31 && H >= 1 && D >= 8 && D % 8 == 0 &&
                      P >= 1 && hp >= 1 && P * hp >= H && ld % 8 == 0 && ldx % 8 == 0,
                  "prism_norm_rope_pack_bwd: bad sizes");
  PRISM_CHECK_ARG(aligned16(g) && aligned16(dx) && (x == nullptr || aligned16(x)) &&
                      (gamma == nullptr || aligned16(gamma)) && (workspace == nullptr || aligned16(workspace)),
                  "prism_norm_rope_pack_bwd: tensors must be 16-byte aligned");
  if (S == 0) return PRISM_OK;
  const int C = H * D, nv = C / 8;
  const int64_t tiles = (S + kProdTileRows - 1) / kProdTileRows;
  PRISM_CHECK_ARG(tiles <= 65535, "prism_norm_rope_pack_bwd: %lld rows exceed the tile grid", (long long)S);
  float* dot = norm ? (float*)workspace : nullptr;
  float* part = norm ? (float*)workspace + ((S + 63) / 64) * 64 : nullptr;
  if (norm) {
    norm_rope_dot_kernel<<<(unsigned)((S * 32 + 255) / 256), 256, 0, stream>>>(
        (const __nv_bfloat16*)g, (const __nv_bfloat16*)x, ld, S, S_pack, H, D, hp, gamma,
        (const float4*)rope_ff, dot);
    PRISM_CHECK_LAUNCH("prism_norm_rope_pack_bwd/dot");
  }
  norm_rope_dx_kernel<<<dim3((unsigned)((nv + kProdThreads - 1) / kProdThreads), (unsigned)tiles),
                        kProdThreads, 0, stream>>>(
      (const __nv_bfloat16*)g, (const __nv_bfloat16*)x, ld, S, S_pack, H, D, hp, gamma, rstd, dot,
      (const float4*)rope_ff,
      norm, (__nv_bfloat16*)dx, ldx, part);
  PRISM_CHECK_LAUNCH("prism_norm_rope_pack_bwd/dx");
  if (norm) {
    // dgamma: tiles partial rows -> <= 64 groups -> 1 (fixed order)
    const int64_t per = (tiles + 63) / 64;
    const int64_t groups = (tiles + per - 1) / per;
    float* part2 = part + tiles * C;
    column_sum_kernel<<<dim3((C + 255) / 256, (unsigned)groups), 256, 0, stream>>>(part, tiles, per, C, part2);
    column_sum_kernel<<<dim3((C + 255) / 256, 1), 256, 0, stream>>>(part2, groups, groups, C, dgamma);
    PRISM_CHECK_LAUNCH("prism_norm_rope_pack_bwd/dgamma");
  }
  return PRISM_OK;
}

}  // extern "C"
