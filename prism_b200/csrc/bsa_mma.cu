// Block-sparse attention forward / backward with warp-level mma.sync tensor
// core tiles (bf16 in, fp32 accumulate).  This is the portable path of the
// library: every CTA owns a PAIR of 64-row tiles (128 rows, the natural
// tcgen05 M) and walks the union of the two tiles' bitmap rows; warps of the
// half that did not select a tile skip it, so no FLOP is spent on unselected
// (q tile, k tile) pairs.
//
// Numerics follow the reference Triton kernels
// (flash_attn_bsa_varlen_mask.py:193-319 forward, :564-704 dK/dV, :881-1014 dQ,
// common.py:94-111 delta):
//   * scores in log2 units: s * (sm_scale * 1.44269504), online softmax with
//     m = -inf, l = 1 initial state and alpha = 1 when the new max is -inf;
//   * masked keys get p = 0 (kv_valid_mask);
//   * lse stored in natural-log units (M * ln2), read back as lse / ln2;
//   * dK *= sm_scale, dQ *= sm_scale (the reference folds sm_scale / ln2 into
//     a bf16 copy of K and multiplies dQ by ln2; here the scale is applied to
//     the fp32 scores instead, which rounds K once less).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "prism_common.cuh"

namespace prism {
namespace mma {

constexpr float kLog2e = 1.44269504f;
constexpr float kLn2 = 0.6931471824645996f;
constexpr float kRcpLn2 = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Row-major [rows][D] bf16 tile in shared memory, 16-byte chunks XOR-swizzled
// within groups of 8 so that ldmatrix rows hit distinct banks.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  const int sw = (chunk & ~7) | ((chunk ^ row) & 7);
  return (uint32_t)(row * D * 2 + sw * 16);
}

// cp.async a [rows][D] tile from global rows (row stride D elements).
template <int D, int ROWS, int NT>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g) {
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    cp_async16(sbase + tile_off<D>(r, c), g + (int64_t)r * D + c * 8);
  }
}

// Union iterator over two bitmap rows in shared memory.
struct UnionIter {
  const uint32_t* ra;
  const uint32_t* rb;
  int wq, wi;
  uint32_t cur;
  __device__ void init(const uint32_t* a, const uint32_t* b, int n) {
    ra = a;
    rb = b;
    wq = n;
    wi = 0;
    cur = n > 0 ? (a[0] | b[0]) : 0u;
  }
  // returns tile index or -1; sel = bit0: first row selected, bit1: second
  __device__ int next(int& sel) {
    while (cur == 0u) {
      if (++wi >= wq) return -1;
      cur = ra[wi] | rb[wi];
    }
    const int b = __ffs(cur) - 1;
    cur &= cur - 1u;
    sel = (int)((ra[wi] >> b) & 1u) | ((int)((rb[wi] >> b) & 1u) << 1);
    return wi * 32 + b;
  }
};

// =================================================================== forward
template <int D>
__global__ void __launch_bounds__(256, 1)
    fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
               const __nv_bfloat16* __restrict__ v, int64_t S, int wq, float qk_scale,
               const uint32_t* __restrict__ bits_q, const uint64_t* __restrict__ tile_bits,
               __nv_bfloat16* __restrict__ o, __nv_bfloat16* __restrict__ o_lo,
               float* __restrict__ lse) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int pair = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 2;
  const int64_t n_tiles = S / 64;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 128 * D * 2;
  uint8_t* sV = sK + 2 * 64 * D * 2;
  uint32_t* sRow = reinterpret_cast<uint32_t*>(sV + 2 * 64 * D * 2);
  const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
  const int64_t hbase = (int64_t)h * S * D;
  const int64_t row0 = (int64_t)pair * 128;

  for (int i = threadIdx.x; i < 2 * wq; i += 256) {
    const int64_t qt = 2 * (int64_t)pair + (i >= wq);
    sRow[i] = bits_q[((int64_t)h * n_tiles + qt) * wq + (i % wq)];
  }
  load_tile<D, 128, 256>(aQ, q + hbase + row0 * D);
  cp_async_commit();
  __syncthreads();

  UnionIter it;
  it.init(sRow, sRow + wq, wq);
  int sel_cur = 0;
  int cur = it.next(sel_cur);
  if (cur >= 0) {
    load_tile<D, 64, 256>(aK, k + hbase + (int64_t)cur * 64 * D);
    load_tile<D, 64, 256>(aV, v + hbase + (int64_t)cur * 64 * D);
  }
  cp_async_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 1.0f, l1 = 1.0f;
  const int g = lane >> 2, tq = lane & 3;
  int stage = 0;

  while (cur >= 0) {
    int sel_nxt = 0;
    const int nxt = it.next(sel_nxt);
    if (nxt >= 0) {
      load_tile<D, 64, 256>(aK + (stage ^ 1) * 64 * D * 2, k + hbase + (int64_t)nxt * 64 * D);
      load_tile<D, 64, 256>(aV + (stage ^ 1) * 64 * D * 2, v + hbase + (int64_t)nxt * 64 * D);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    if ((sel_cur >> half) & 1) {
      const uint32_t kb = aK + stage * 64 * D * 2, vb = aV + stage * 64 * D * 2;
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, aQ + tile_off<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
#pragma unroll
        for (int nb2 = 0; nb2 < 4; ++nb2) {
          uint32_t b[4];
          ldsm_x4(b, kb + tile_off<D>(nb2 * 16 + (lane & 7) + ((lane >> 4) << 3),
                                      kk * 2 + ((lane >> 3) & 1)));
          mma16816(s[2 * nb2], a, b);
          mma16816(s[2 * nb2 + 1], a, b + 2);
        }
      }
      const uint64_t vbits = tile_bits[cur];
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nb * 8 + tq * 2 + j;
          if (!((vbits >> col) & 1ull)) {
            s[nb][j] = -INFINITY;
            s[nb][2 + j] = -INFINITY;
          }
          mx0 = fmaxf(mx0, s[nb][j]);
          mx1 = fmaxf(mx1, s[nb][2 + j]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0 * qk_scale), mn1 = fmaxf(m1, mx1 * qk_scale);
      const float al0 = (mn0 == -INFINITY) ? 1.0f : ex2(m0 - mn0);
      const float al1 = (mn1 == -INFINITY) ? 1.0f : ex2(m1 - mn1);
      float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nb * 8 + tq * 2 + j;
          const bool ok = (vbits >> col) & 1ull;
          const float p0 = ok ? ex2(s[nb][j] * qk_scale - mn0) : 0.0f;
          const float p1 = ok ? ex2(s[nb][2 + j] * qk_scale - mn1) : 0.0f;
          s[nb][j] = p0;
          s[nb][2 + j] = p1;
          rs0 += p0;
          rs1 += p1;
        }
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        acc[i][0] *= al0;
        acc[i][1] *= al0;
        acc[i][2] *= al1;
        acc[i][3] *= al1;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int db = 0; db < D / 16; ++db) {
          uint32_t b[4];
          ldsm_x4_t(b, vb + tile_off<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                         db * 2 + (lane >> 4)));
          mma16816(acc[2 * db], a, b);
          mma16816(acc[2 * db + 1], a, b + 2);
        }
      }
    }
    __syncthreads();
    stage ^= 1;
    cur = nxt;
    sel_cur = sel_nxt;
  }
  cp_async_wait<0>();

  // epilogue
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  const int64_t r0 = row0 + warp * 16 + g;
  __nv_bfloat16* o0 = o + hbase + r0 * D;
  __nv_bfloat16* o1 = o0 + 8 * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int c = i * 8 + tq * 2;
    const float x0 = acc[i][0] * inv0, x1 = acc[i][1] * inv0;
    const float x2 = acc[i][2] * inv1, x3 = acc[i][3] * inv1;
    const uint32_t h01 = pack_bf16(x0, x1), h23 = pack_bf16(x2, x3);
    *reinterpret_cast<uint32_t*>(o0 + c) = h01;
    *reinterpret_cast<uint32_t*>(o1 + c) = h23;
    if (o_lo != nullptr) {
      // bf16 rounding residual: O = hi + lo to ~16 mantissa bits, so that the
      // backward's delta = rowsum(O * dO) does not inherit O's bf16 rounding
      const int64_t off0 = (o0 - o) + c, off1 = (o1 - o) + c;
      *reinterpret_cast<uint32_t*>(o_lo + off0) =
          pack_bf16(x0 - __uint_as_float(h01 << 16), x1 - __uint_as_float(h01 & 0xffff0000u));
      *reinterpret_cast<uint32_t*>(o_lo + off1) =
          pack_bf16(x2 - __uint_as_float(h23 << 16), x3 - __uint_as_float(h23 & 0xffff0000u));
    }
  }
  if (tq == 0) {
    lse[(int64_t)h * S + r0] = (m0 + __log2f(l0)) * kLn2;
    lse[(int64_t)h * S + r0 + 8] = (m1 + __log2f(l1)) * kLn2;
  }
}

// ================================================================ preprocess
// delta[h][s] = sum_d O * dO (fp32), one warp per row.
// With o_lo (the forward's rounding residual) the row uses O = hi + lo.
template <int D>
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ o_lo,
                             const __nv_bfloat16* __restrict__ dout, int64_t rows,
                             float* __restrict__ delta) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float acc = 0.0f;
#pragma unroll
  for (int c = lane * 2; c < D; c += 64) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(o + r * D + c);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(dout + r * D + c);
    float a0 = __low2float(a), a1 = __high2float(a);
    if (o_lo != nullptr) {
      const __nv_bfloat162 l = *reinterpret_cast<const __nv_bfloat162*>(o_lo + r * D + c);
      a0 += __low2float(l);
      a1 += __high2float(l);
    }
    acc += a0 * __low2float(b) + a1 * __high2float(b);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[r] = acc;
}

// ================================================================== dK / dV
// CTA = 128 keys (key tiles 2p, 2p+1); loops over the union of the q tiles that
// selected either key tile (bits_k rows).
template <int D>
__global__ void __launch_bounds__(256, 1)
    dkdv_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ dout,
                const float* __restrict__ lse, const float* __restrict__ delta, int64_t S, int wq,
                float qk_scale, float sm_scale, const uint32_t* __restrict__ bits_k,
                const uint64_t* __restrict__ tile_bits, __nv_bfloat16* __restrict__ dk,
                __nv_bfloat16* __restrict__ dv) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int pair = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 2;
  const int64_t n_tiles = S / 64;
  uint8_t* sK = smem;
  uint8_t* sV = sK + 128 * D * 2;
  uint8_t* sQ = sV + 128 * D * 2;       // 2 stages x 64 rows
  uint8_t* sDO = sQ + 2 * 64 * D * 2;   // 2 stages x 64 rows
  float* sM = reinterpret_cast<float*>(sDO + 2 * 64 * D * 2);  // 2 x 64
  float* sDl = sM + 128;                                        // 2 x 64
  uint32_t* sRow = reinterpret_cast<uint32_t*>(sDl + 128);
  const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
  const int64_t hbase = (int64_t)h * S * D;
  const int64_t key0 = (int64_t)pair * 128;

  for (int i = threadIdx.x; i < 2 * wq; i += 256) {
    const int64_t kt = 2 * (int64_t)pair + (i >= wq);
    sRow[i] = bits_k[((int64_t)h * n_tiles + kt) * wq + (i % wq)];
  }
  load_tile<D, 128, 256>(aK, k + hbase + key0 * D);
  load_tile<D, 128, 256>(aV, v + hbase + key0 * D);
  cp_async_commit();
  __syncthreads();

  UnionIter it;
  it.init(sRow, sRow + wq, wq);
  int sel_cur = 0;
  int cur = it.next(sel_cur);
  auto issue = [&](int st, int qt) {
    load_tile<D, 64, 256>(aQ + st * 64 * D * 2, q + hbase + (int64_t)qt * 64 * D);
    load_tile<D, 64, 256>(aDO + st * 64 * D * 2, dout + hbase + (int64_t)qt * 64 * D);
    if (threadIdx.x < 64) {
      const int64_t r = (int64_t)h * S + (int64_t)qt * 64 + threadIdx.x;
      sM[st * 64 + threadIdx.x] = lse[r] * kRcpLn2;
      sDl[st * 64 + threadIdx.x] = delta[r];
    }
  };
  if (cur >= 0) issue(0, cur);
  cp_async_commit();

  float adk[D / 8][4], adv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) adk[i][j] = adv[i][j] = 0.0f;
  const int g = lane >> 2, tq = lane & 3;
  const uint64_t kbits = tile_bits[2 * pair + half];
  const int kl0 = (warp & 3) * 16 + g;  // key index within its 64-key tile
  const bool kv0 = (kbits >> kl0) & 1ull, kv1 = (kbits >> (kl0 + 8)) & 1ull;
  int stage = 0;

  while (cur >= 0) {
    int sel_nxt = 0;
    const int nxt = it.next(sel_nxt);
    __syncthreads();  // stage^1 (and its M / delta) no longer read
    if (nxt >= 0) issue(stage ^ 1, nxt);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    if ((sel_cur >> half) & 1) {
      const uint32_t qb = aQ + stage * 64 * D * 2, db = aDO + stage * 64 * D * 2;
      const float* m = sM + stage * 64;
      const float* dl = sDl + stage * 64;
      // S^T = K Q^T  (16 keys x 64 queries)
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, aK + tile_off<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
#pragma unroll
        for (int nb2 = 0; nb2 < 4; ++nb2) {
          uint32_t b[4];
          ldsm_x4(b, qb + tile_off<D>(nb2 * 16 + (lane & 7) + ((lane >> 4) << 3),
                                      kk * 2 + ((lane >> 3) & 1)));
          mma16816(s[2 * nb2], a, b);
          mma16816(s[2 * nb2 + 1], a, b + 2);
        }
      }
      // P^T
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float mq = m[nb * 8 + tq * 2 + j];
          s[nb][j] = kv0 ? ex2(s[nb][j] * qk_scale - mq) : 0.0f;
          s[nb][2 + j] = kv1 ? ex2(s[nb][2 + j] * qk_scale - mq) : 0.0f;
        }
      }
      // dP^T = V dO^T
      float dp[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, aV + tile_off<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
#pragma unroll
        for (int nb2 = 0; nb2 < 4; ++nb2) {
          uint32_t b[4];
          ldsm_x4(b, db + tile_off<D>(nb2 * 16 + (lane & 7) + ((lane >> 4) << 3),
                                      kk * 2 + ((lane >> 3) & 1)));
          mma16816(dp[2 * nb2], a, b);
          mma16816(dp[2 * nb2 + 1], a, b + 2);
        }
      }
      // dV += P^T dO ; dS^T = P^T (dP^T - delta) ; dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ap[4], as[4];
        ap[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        ap[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        ap[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        ap[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        float ds[2][4];
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int nb = 2 * kk + hb;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float dq = dl[nb * 8 + tq * 2 + j];
            ds[hb][j] = s[nb][j] * (dp[nb][j] - dq);
            ds[hb][2 + j] = s[nb][2 + j] * (dp[nb][2 + j] - dq);
          }
        }
        as[0] = pack_bf16(ds[0][0], ds[0][1]);
        as[1] = pack_bf16(ds[0][2], ds[0][3]);
        as[2] = pack_bf16(ds[1][0], ds[1][1]);
        as[3] = pack_bf16(ds[1][2], ds[1][3]);
#pragma unroll
        for (int dbk = 0; dbk < D / 16; ++dbk) {
          uint32_t b[4];
          ldsm_x4_t(b, db + tile_off<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                         dbk * 2 + (lane >> 4)));
          mma16816(adv[2 * dbk], ap, b);
          mma16816(adv[2 * dbk + 1], ap, b + 2);
          ldsm_x4_t(b, qb + tile_off<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                         dbk * 2 + (lane >> 4)));
          mma16816(adk[2 * dbk], as, b);
          mma16816(adk[2 * dbk + 1], as, b + 2);
        }
      }
    }
    stage ^= 1;
    cur = nxt;
    sel_cur = sel_nxt;
  }
  cp_async_wait<0>();

  const int64_t r0 = key0 + warp * 16 + g;
  __nv_bfloat16* k0 = dk + hbase + r0 * D;
  __nv_bfloat16* v0 = dv + hbase + r0 * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int c = i * 8 + tq * 2;
    *reinterpret_cast<uint32_t*>(k0 + c) = pack_bf16(adk[i][0] * sm_scale, adk[i][1] * sm_scale);
    *reinterpret_cast<uint32_t*>(k0 + 8 * D + c) = pack_bf16(adk[i][2] * sm_scale, adk[i][3] * sm_scale);
    *reinterpret_cast<uint32_t*>(v0 + c) = pack_bf16(adv[i][0], adv[i][1]);
    *reinterpret_cast<uint32_t*>(v0 + 8 * D + c) = pack_bf16(adv[i][2], adv[i][3]);
  }
}

// ======================================================================= dQ
template <int D>
__global__ void __launch_bounds__(256, 1)
    dq_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
              const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ dout,
              const float* __restrict__ lse, const float* __restrict__ delta, int64_t S, int wq,
              float qk_scale, float sm_scale, const uint32_t* __restrict__ bits_q,
              const uint64_t* __restrict__ tile_bits, __nv_bfloat16* __restrict__ dq) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int pair = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 2;
  const int64_t n_tiles = S / 64;
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + 128 * D * 2;
  uint8_t* sK = sDO + 128 * D * 2;
  uint8_t* sV = sK + 2 * 64 * D * 2;
  uint32_t* sRow = reinterpret_cast<uint32_t*>(sV + 2 * 64 * D * 2);
  const uint32_t aQ = smem_u32(sQ), aDO = smem_u32(sDO), aK = smem_u32(sK), aV = smem_u32(sV);
  const int64_t hbase = (int64_t)h * S * D;
  const int64_t row0 = (int64_t)pair * 128;

  for (int i = threadIdx.x; i < 2 * wq; i += 256) {
    const int64_t qt = 2 * (int64_t)pair + (i >= wq);
    sRow[i] = bits_q[((int64_t)h * n_tiles + qt) * wq + (i % wq)];
  }
  load_tile<D, 128, 256>(aQ, q + hbase + row0 * D);
  load_tile<D, 128, 256>(aDO, dout + hbase + row0 * D);
  cp_async_commit();
  __syncthreads();

  const int g = lane >> 2, tq = lane & 3;
  const int64_t r0 = row0 + warp * 16 + g;
  const float mr0 = lse[(int64_t)h * S + r0] * kRcpLn2, mr1 = lse[(int64_t)h * S + r0 + 8] * kRcpLn2;
  const float dl0 = delta[(int64_t)h * S + r0], dl1 = delta[(int64_t)h * S + r0 + 8];

  UnionIter it;
  it.init(sRow, sRow + wq, wq);
  int sel_cur = 0;
  int cur = it.next(sel_cur);
  if (cur >= 0) {
    load_tile<D, 64, 256>(aK, k + hbase + (int64_t)cur * 64 * D);
    load_tile<D, 64, 256>(aV, v + hbase + (int64_t)cur * 64 * D);
  }
  cp_async_commit();

  float adq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) adq[i][0] = adq[i][1] = adq[i][2] = adq[i][3] = 0.0f;
  int stage = 0;
  while (cur >= 0) {
    int sel_nxt = 0;
    const int nxt = it.next(sel_nxt);
    if (nxt >= 0) {
      load_tile<D, 64, 256>(aK + (stage ^ 1) * 64 * D * 2, k + hbase + (int64_t)nxt * 64 * D);
      load_tile<D, 64, 256>(aV + (stage ^ 1) * 64 * D * 2, v + hbase + (int64_t)nxt * 64 * D);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if ((sel_cur >> half) & 1) {
      const uint32_t kb = aK + stage * 64 * D * 2, vb = aV + stage * 64 * D * 2;
      float s[8][4], dp[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4], ad[4];
        ldsm_x4(a, aQ + tile_off<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
        ldsm_x4(ad, aDO + tile_off<D>(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
#pragma unroll
        for (int nb2 = 0; nb2 < 4; ++nb2) {
          uint32_t b[4];
          const int rr = nb2 * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int cc = kk * 2 + ((lane >> 3) & 1);
          ldsm_x4(b, kb + tile_off<D>(rr, cc));
          mma16816(s[2 * nb2], a, b);
          mma16816(s[2 * nb2 + 1], a, b + 2);
          ldsm_x4(b, vb + tile_off<D>(rr, cc));
          mma16816(dp[2 * nb2], ad, b);
          mma16816(dp[2 * nb2 + 1], ad, b + 2);
        }
      }
      const uint64_t vbits = tile_bits[cur];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nb * 8 + tq * 2 + j;
          const bool ok = (vbits >> col) & 1ull;
          const float p0 = ok ? ex2(s[nb][j] * qk_scale - mr0) : 0.0f;
          const float p1 = ok ? ex2(s[nb][2 + j] * qk_scale - mr1) : 0.0f;
          s[nb][j] = p0 * (dp[nb][j] - dl0);
          s[nb][2 + j] = p1 * (dp[nb][2 + j] - dl1);
        }
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int dbk = 0; dbk < D / 16; ++dbk) {
          uint32_t b[4];
          ldsm_x4_t(b, kb + tile_off<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                         dbk * 2 + (lane >> 4)));
          mma16816(adq[2 * dbk], a, b);
          mma16816(adq[2 * dbk + 1], a, b + 2);
        }
      }
    }
    __syncthreads();
    stage ^= 1;
    cur = nxt;
    sel_cur = sel_nxt;
  }
  cp_async_wait<0>();
  __nv_bfloat16* q0 = dq + hbase + r0 * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int c = i * 8 + tq * 2;
    *reinterpret_cast<uint32_t*>(q0 + c) = pack_bf16(adq[i][0] * sm_scale, adq[i][1] * sm_scale);
    *reinterpret_cast<uint32_t*>(q0 + 8 * D + c) = pack_bf16(adq[i][2] * sm_scale, adq[i][3] * sm_scale);
  }
}

template <int D>
size_t fwd_smem(int wq) { return (size_t)(128 + 4 * 64) * D * 2 + 2 * wq * 4; }
template <int D>
size_t dkdv_smem(int wq) { return (size_t)(256 + 4 * 64) * D * 2 + 4 * 128 * 4 + 2 * wq * 4; }
template <int D>
size_t dq_smem(int wq) { return (size_t)(256 + 4 * 64) * D * 2 + 2 * wq * 4; }

template <int D>
prism_status_t launch_fwd(const void* q, const void* k, const void* v, int heads, int64_t S,
                          float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits, void* o,
                          void* o_lo, float* lse, cudaStream_t stream) {
  const int64_t n_tiles = S / 64;
  const int wq = (int)((n_tiles + 31) / 32);
  const size_t sm = fwd_smem<D>(wq);
  PRISM_CHECK_ARG(sm <= 227 * 1024, "prism_bsa_fwd: sequence too long for the bitmap row cache");
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_fwd: smem attribute");
  fwd_kernel<D><<<dim3((unsigned)(n_tiles / 2), heads), 256, sm, stream>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, S, wq,
      sm_scale * kLog2e, bits_q, tile_bits, (__nv_bfloat16*)o, (__nv_bfloat16*)o_lo, lse);
  PRISM_CHECK_LAUNCH("prism_bsa_fwd");
  return PRISM_OK;
}

template <int D>
prism_status_t launch_delta(const void* o, const void* o_lo, const void* dout, int heads, int64_t S,
                            float* delta, cudaStream_t stream) {
  const int64_t rows = (int64_t)heads * S;
  delta_kernel<D><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, stream>>>(
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)o_lo, (const __nv_bfloat16*)dout, rows, delta);
  PRISM_CHECK_LAUNCH("prism_bsa_bwd_delta");
  return PRISM_OK;
}

template <int D>
prism_status_t launch_dkdv(const void* q, const void* k, const void* v, const void* dout,
                           const float* lse, const float* delta, int heads, int64_t S,
                           float sm_scale, const uint32_t* bits_k, const uint64_t* tile_bits,
                           void* dk, void* dv, cudaStream_t stream) {
  const int64_t n_tiles = S / 64;
  const int wq = (int)((n_tiles + 31) / 32);
  const size_t sm = dkdv_smem<D>(wq);
  PRISM_CHECK_ARG(sm <= 227 * 1024, "prism_bsa_bwd: sequence too long for the bitmap row cache");
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(dkdv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_bwd: smem attribute");
  dkdv_kernel<D><<<dim3((unsigned)(n_tiles / 2), heads), 256, sm, stream>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
      (const __nv_bfloat16*)dout, lse, delta, S, wq, sm_scale * (float)kRcpLn2, sm_scale, bits_k,
      tile_bits, (__nv_bfloat16*)dk, (__nv_bfloat16*)dv);
  PRISM_CHECK_LAUNCH("prism_bsa_bwd_dkdv");
  return PRISM_OK;
}

template <int D>
prism_status_t launch_dq(const void* q, const void* k, const void* v, const void* dout,
                         const float* lse, const float* delta, int heads, int64_t S,
                         float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                         void* dq, cudaStream_t stream) {
  const int64_t n_tiles = S / 64;
  const int wq = (int)((n_tiles + 31) / 32);
  const size_t sm = dq_smem<D>(wq);
  PRISM_CHECK_ARG(sm <= 227 * 1024, "prism_bsa_bwd: sequence too long for the bitmap row cache");
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_bwd: smem attribute");
  dq_kernel<D><<<dim3((unsigned)(n_tiles / 2), heads), 256, sm, stream>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
      (const __nv_bfloat16*)dout, lse, delta, S, wq, sm_scale * (float)kRcpLn2, sm_scale, bits_q,
      tile_bits, (__nv_bfloat16*)dq);
  PRISM_CHECK_LAUNCH("prism_bsa_bwd_dq");
  return PRISM_OK;
}

}  // namespace mma
}  // namespace prism

using namespace prism;

extern "C" {

prism_status_t prism_bsa_fwd(const void* q, const void* k, const void* v, int heads, int64_t S,
                             int D, float sm_scale, const uint32_t* bits_q,
                             const uint64_t* tile_bits, void* o, void* o_lo, float* lse,
                             cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && bits_q && tile_bits && o && lse, "prism_bsa_fwd: null pointer");
  PRISM_CHECK_ARG(S > 0 && S % 128 == 0 && heads >= 1, "prism_bsa_fwd: S must be a positive multiple of 128");
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o), "prism_bsa_fwd: tensors must be 16-byte aligned");
  PRISM_CHECK_ARG(o_lo == nullptr || aligned16(o_lo), "prism_bsa_fwd: o_lo must be 16-byte aligned");
  if (D == 128) return mma::launch_fwd<128>(q, k, v, heads, S, sm_scale, bits_q, tile_bits, o, o_lo, lse, stream);
  if (D == 64) return mma::launch_fwd<64>(q, k, v, heads, S, sm_scale, bits_q, tile_bits, o, o_lo, lse, stream);
  set_error("prism_bsa_fwd: head dim %d not supported (64, 128)", D);
  return PRISM_ERR_UNSUPPORTED;
}

size_t prism_bsa_bwd_workspace_bytes(int heads, int64_t S) {
  return (size_t)heads * (size_t)S * sizeof(float);
}

#define PRISM_BWD_COMMON_CHECKS(name)                                                              \
  PRISM_CHECK_ARG(S > 0 && S % 128 == 0 && heads >= 1, name ": S must be a positive multiple of 128"); \
  PRISM_CHECK_ARG(D == 64 || D == 128, name ": head dim %d not supported (64, 128)", D)

prism_status_t prism_bsa_bwd_delta(const void* o, const void* o_lo, const void* dout, int heads,
                                   int64_t S, int D, float* delta, cudaStream_t stream) {
  PRISM_CHECK_ARG(o && dout && delta, "prism_bsa_bwd_delta: null pointer");
  PRISM_BWD_COMMON_CHECKS("prism_bsa_bwd_delta");
  return D == 128 ? mma::launch_delta<128>(o, o_lo, dout, heads, S, delta, stream)
                  : mma::launch_delta<64>(o, o_lo, dout, heads, S, delta, stream);
}

prism_status_t prism_bsa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout,
                                  const float* lse, const float* delta, int heads, int64_t S, int D,
                                  float sm_scale, const uint32_t* bits_k, const uint64_t* tile_bits,
                                  void* dk, void* dv, cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && dout && lse && delta && bits_k && tile_bits && dk && dv,
                  "prism_bsa_bwd_dkdv: null pointer");
  PRISM_BWD_COMMON_CHECKS("prism_bsa_bwd_dkdv");
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dout) && aligned16(dk) && aligned16(dv),
                  "prism_bsa_bwd_dkdv: tensors must be 16-byte aligned");
  return D == 128 ? mma::launch_dkdv<128>(q, k, v, dout, lse, delta, heads, S, sm_scale, bits_k, tile_bits, dk, dv, stream)
                  : mma::launch_dkdv<64>(q, k, v, dout, lse, delta, heads, S, sm_scale, bits_k, tile_bits, dk, dv, stream);
}

prism_status_t prism_bsa_bwd_dq(const void* q, const void* k, const void* v, const void* dout,
                                const float* lse, const float* delta, int heads, int64_t S, int D,
                                float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                                void* dq, cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && dout && lse && delta && bits_q && tile_bits && dq, "prism_bsa_bwd_dq: null pointer");
  PRISM_BWD_COMMON_CHECKS("prism_bsa_bwd_dq");
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dout) && aligned16(dq),
                  "prism_bsa_bwd_dq: tensors must be 16-byte aligned");
  return D == 128 ? mma::launch_dq<128>(q, k, v, dout, lse, delta, heads, S, sm_scale, bits_q, tile_bits, dq, stream)
                  : mma::launch_dq<64>(q, k, v, dout, lse, delta, heads, S, sm_scale, bits_q, tile_bits, dq, stream);
}

prism_status_t prism_bsa_bwd(const void* q, const void* k, const void* v, const void* o,
                             const void* o_lo, const void* dout, const float* lse, int heads,
                             int64_t S, int D,
                             float sm_scale, const uint32_t* bits_q, const uint32_t* bits_k,
                             const uint64_t* tile_bits, void* workspace, void* dq, void* dk,
                             void* dv, cudaStream_t stream) {
  PRISM_CHECK_ARG(workspace, "prism_bsa_bwd: null pointer");
  float* delta = (float*)workspace;
  prism_status_t st = prism_bsa_bwd_delta(o, o_lo, dout, heads, S, D, delta, stream);
  if (st != PRISM_OK) return st;
  st = prism_bsa_bwd_dkdv(q, k, v, dout, lse, delta, heads, S, D, sm_scale, bits_k, tile_bits, dk, dv, stream);
  if (st != PRISM_OK) return st;
  return prism_bsa_bwd_dq(q, k, v, dout, lse, delta, heads, S, D, sm_scale, bits_q, tile_bits, dq, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------
// Backward without any device allocation (prism_bsa_bwd_noalloc).
//
// The only scratch the backward needs is delta[h][s] (one float per query
// row).  Here it lives in a file-scope device array of a fixed size, so the
// caller passes inputs and outputs only.  The array is part of this library's
// device image: every GPU that loads the library reserves it until the
// process exits.  Host code cannot use the array's name as a device address
// (on the host it names a stand-in object), so its real address is looked up
// with cudaGetSymbolAddress, once per device, with that device current, on
// the first call made on that device.
namespace prism {
namespace mma {
static __device__ __align__(256) float g_noalloc_delta[PRISM_BSA_BWD_NOALLOC_MAX_ROWS];
}  // namespace mma

static std::mutex g_noalloc_mu;
static float* g_noalloc_addr[128] = {nullptr};

static prism_status_t noalloc_scratch(float** out) {
  int dev = -1;
  PRISM_CHECK_CUDA(cudaGetDevice(&dev), "prism_bsa_bwd_noalloc: cudaGetDevice");
  PRISM_CHECK_ARG(dev >= 0 && dev < 128, "prism_bsa_bwd_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, mma::g_noalloc_delta);
    if (e != cudaSuccess || p == nullptr) {
      set_error("prism_bsa_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return PRISM_ERR_CUDA;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[dev];
  return PRISM_OK;
}
}  // namespace prism

extern "C" prism_status_t prism_bsa_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* o_lo, const void* dout,
    const float* lse, int heads, int64_t S, int D, float sm_scale, const uint32_t* bits_q,
    const uint32_t* bits_k, const uint64_t* tile_bits, void* dq, void* dk, void* dv,
    cudaStream_t stream) {
  PRISM_CHECK_ARG(heads >= 1 && S > 0, "prism_bsa_bwd_noalloc: heads and S must be positive");
  PRISM_CHECK_ARG((uint64_t)heads * (uint64_t)S <= (uint64_t)PRISM_BSA_BWD_NOALLOC_MAX_ROWS,
                  "prism_bsa_bwd_noalloc: heads*S = %lld query rows exceed the built-in scratch "
                  "of %u rows; use prism_bsa_bwd with a caller-provided workspace",
                  (long long)heads * (long long)S, (unsigned)PRISM_BSA_BWD_NOALLOC_MAX_ROWS);
  float* delta = nullptr;
  const prism_status_t st0 = noalloc_scratch(&delta);
  if (st0 != PRISM_OK) return st0;
  // Every delta row is written by the first stage before the other two read
  // it, so nothing left in the array by an earlier call is ever used.
  prism_status_t st = prism_bsa_bwd_delta(o, o_lo, dout, heads, S, D, delta, stream);
  if (st != PRISM_OK) return st;
  st = prism_bsa_bwd_dkdv(q, k, v, dout, lse, delta, heads, S, D, sm_scale, bits_k, tile_bits, dk, dv, stream);
  if (st != PRISM_OK) return st;
  return prism_bsa_bwd_dq(q, k, v, dout, lse, delta, heads, S, D, sm_scale, bits_q, tile_bits, dq, stream);
}
