// Block-sparse attention forward / backward on the sm_100a tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA in 128B-swizzled
// shared memory).
//
// Work decomposition.  Tokens are in tile order (64-token tiles).  Selections
// are bitmaps: bits_q[h][q tile] marks the key tiles a query tile attends,
// bits_k is its transpose.
//
//   forward   CTA = 256 queries (tiles 4p..4p+3) as two groups of 128 rows;
//             per step a pair of key tiles (N = 128) computed by one or both
//             groups (FwdSched): S = Q K^T -> TMEM, online softmax in
//             registers (one thread per query row), P (bf16) written over S in
//             TMEM, O += P V with P read from TMEM.
//   dK / dV   CTA = 128 keys (tiles 2p, 2p+1); per step two query tiles (N =
//             128) of the union of the two key tiles' transposed rows:
//             S^T = K Q^T, dP^T = V dO^T -> TMEM, P^T and dS^T written over
//             them in TMEM, dV += P^T dO, dK += dS^T Q.
//   dQ        CTA = 128 queries (tiles 2p, 2p+1); per step a pair of key tiles
//             of the union of the two rows: S, dP -> TMEM, dS -> TMEM,
//             dQ += dS K.
// Rows of a tile that did not select a key tile get p = 0 for it, so every
// kernel computes exactly the per-tile sparse attention of the reference.
//
// Warp roles (320 threads): warps 0-7 = softmax / epilogue (thread i of a
// warpgroup owns TMEM lane i), warp 8 = TMA producer, warp 9 = MMA issuer
// (one thread) and TMEM owner.  Producer, MMA issuer and softmax warps all
// walk the same tile sequence from the bitmaps, so they agree on it without
// exchanging it.
//
// Numerics follow the reference Triton kernels
// (hymm/models/modules/block_sparse_attention/flash_attn_bsa_varlen_mask.py:
// 193-319 forward, 564-704 dK/dV, 881-1014 dQ; common.py:94-111 delta):
// scores in log2 units s * sm_scale * log2(e); initial state m = -inf, l = 1;
// masked keys get p = 0; lse stored in natural-log units; dK and dQ scaled by
// sm_scale.  The forward keeps a running maximum that is only raised when the
// new block maximum exceeds it by more than 2^8 (the rescale of O in TMEM is
// then rare); p = exp2(s - m) <= 256 stays exact in fp32 and is rounded to
// bf16 for P V exactly as the reference rounds p.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <mutex>

#include "prism_common.cuh"
#include "sm100.cuh"

namespace prism {
namespace tc {

using namespace sm100;

constexpr float kLn2 = 0.6931471824645996f;
constexpr float kRcpLn2 = 1.4426950408889634f;
// Backward kernels: 8 softmax warps (two warpgroups splitting each step's
// columns) + producer + MMA.
constexpr int kBwdThreads = 320;
constexpr int kBwdProducerWarp = 8;
constexpr int kBwdMmaWarp = 9;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Device error word: 0 = ok, otherwise the code of the first bounded wait that
// gave up (see prism_device_status).
__device__ int g_tc_error = 0;

enum WaitCode : int {
  kErrFwdProducer = 101, kErrFwdMma = 102, kErrFwdSoftmax = 103,
  kErrDkdvProducer = 201, kErrDkdvMma = 202, kErrDkdvSoftmax = 203,
  kErrDqProducer = 301, kErrDqMma = 302, kErrDqSoftmax = 303,
};

// Union iterator over two bitmap rows (global memory, read through the
// read-only cache).  Every role of a CTA runs its own copy and sees the same
// sequence: increasing tile index.
struct UnionIter {
  const uint32_t* ra;
  const uint32_t* rb;
  int wq, wi;
  uint32_t a, b;
  __device__ __forceinline__ void init(const uint32_t* row_a, const uint32_t* row_b, int n) {
    ra = row_a;
    rb = row_b;
    wq = n;
    wi = 0;
    a = n > 0 ? __ldg(ra) : 0u;
    b = n > 0 ? __ldg(rb) : 0u;
  }
  // next tile index, or -1; sel bit 0: first row selected it, bit 1: second row
  __device__ __forceinline__ int next(int& sel) {
    while ((a | b) == 0u) {
      if (++wi >= wq) return -1;
      a = __ldg(ra + wi);
      b = __ldg(rb + wi);
    }
    const int bit = __ffs(a | b) - 1;
    const uint32_t m = 1u << bit;
    sel = ((a & m) ? 1 : 0) | ((b & m) ? 2 : 0);
    a &= ~m;
    b &= ~m;
    return wi * 32 + bit;
  }
};

// Number of tiles in the union of two bitmap rows (the steps a backward CTA takes).
__device__ __forceinline__ int union_count(const uint32_t* ra, const uint32_t* rb, int wq) {
  int c = 0;
  for (int w = 0; w < wq; ++w) c += __popc(__ldg(ra + w) | __ldg(rb + w));
  return c;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Warp-uniform bounded wait (every lane must agree before a .sync.aligned op).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int code) {
  bool ok = mbar_wait(bar, parity, abort_flag, &g_tc_error, code);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) *abort_flag = 1;
  return ok;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }

// 32 * N consecutive TMEM columns of this warp's 32 lanes -> registers (waited).
template <int N>
__device__ __forceinline__ void tmem_load(uint32_t taddr, float (&out)[32 * N]) {
  uint32_t raw[N][32];
#pragma unroll
  for (int c = 0; c < N; ++c) tmem_ld32(taddr + c * 32, raw[c]);
#pragma unroll
  for (int c = 0; c < N; ++c) tmem_wait_ld_dep(raw[c]);
#pragma unroll
  for (int c = 0; c < N; ++c)
#pragma unroll
    for (int i = 0; i < 32; ++i) out[c * 32 + i] = u2f(raw[c][i]);
}

// Request at least this much dynamic shared memory so that a second CTA never
// shares the SM (each CTA allocates 512 TMEM columns, the whole TMEM).
constexpr size_t kMinSmem = 116 * 1024;

// ===================================================================== forward
// CTA = 256 queries = tiles 4p..4p+3, as two groups of 128 rows (g = 0: tiles
// 4p, 4p+1; g = 1: tiles 4p+2, 4p+3) that share one stream of key-tile pairs
// (FwdSched below).  Each group has its own softmax warpgroup, S buffer and
// O accumulator in TMEM, so while one group's softmax runs the tensor core
// works on the other group's products.
// The forward's steps.  The key tiles of the four-row union fall into three
// classes: tiles some row of BOTH groups selected (A), tiles only group 0
// selected (B), only group 1 (C).  At the start of the kernel all threads
// write the three classes' tiles, each in increasing tile order, into one
// shared-memory list (A, then B, then C: build_fwd_lists); each class is then
// paired in list order, and step n is decoded from the three counts in O(1):
//   1. couples: B pair i (mask 1: group 0 computes it), C pair i (mask 2),
//      for i < k = min(pairs B, pairs C) -- the groups alternate on the
//      tensor core as with two-group steps, and no product is spent on key
//      tiles a group did not select;
//   2. the class left over, X (B or C), interleaved with A pairs: A pair i
//      (mask 3), X pair k + i (mask of X), for i < j = min(pairs A, pairs X - k);
//   3. the remaining A pairs, then the remaining X pairs computed by both
//      groups (mask 3; the other group's rows get p = 0), the unpaired A tile
//      (mask 3) and the unpaired B / C tiles (one step, mask 3).
// At the uniform path's 25 % density the four-row union is ~1.8x each group's
// own union; this schedule computes ~1.04x the selected products (dynamic
// path, 85 %: ~1.01x, as before).
struct FwdSched {
  const uint16_t* list;
  int nA, nB, nC, pA, k, j, X, remX, total;
  __device__ __forceinline__ void init(const uint16_t* l, const int* counts) {
    list = l;
    nA = counts[0], nB = counts[1], nC = counts[2];
    pA = nA >> 1;
    const int pB = nB >> 1, pC = nC >> 1;
    k = min(pB, pC);
    X = pB > k ? 1 : 2;
    remX = max(pB, pC) - k;
    j = min(pA, remX);
    total = 2 * k + 2 * j + (pA - j) + (remX - j) + (nA & 1) + (((nB | nC) & 1) ? 1 : 0);
  }
  // tiles of pair i of class c (0 = A, 1 = B, 2 = C)
  __device__ __forceinline__ void pair(int c, int i, int& t0, int& t1) const {
    const uint16_t* b = list + (c == 0 ? 0 : (c == 1 ? nA : nA + nB)) + 2 * i;
    t0 = b[0];
    t1 = b[1];
  }
  __device__ __forceinline__ void step(int n, int& t0, int& t1, int& mask) const {
    if (n < 2 * k) {
      pair((n & 1) ? 2 : 1, n >> 1, t0, t1);
      mask = (n & 1) ? 2 : 1;
      return;
    }
    n -= 2 * k;
    if (n < 2 * j) {
      if (n & 1) {
        pair(X, k + (n >> 1), t0, t1);
        mask = X;
      } else {
        pair(0, n >> 1, t0, t1);
        mask = 3;
      }
      return;
    }
    n -= 2 * j;
    mask = 3;
    if (n < pA - j) {
      pair(0, j + n, t0, t1);
      return;
    }
    n -= pA - j;
    if (n < remX - j) {
      pair(X, k + j + n, t0, t1);
      return;
    }
    n -= remX - j;
    if (nA & 1) {
      if (n == 0) {
        t0 = list[nA - 1];
        t1 = -1;
        return;
      }
      --n;
    }
    const int sb = (nB & 1) ? (int)list[nA + nB - 1] : -1;
    const int sc = (nC & 1) ? (int)list[nA + nB + nC - 1] : -1;
    t0 = sb >= 0 ? sb : sc;
    t1 = sb >= 0 ? sc : -1;
  }
};

// All threads of the CTA: the class lists of FwdSched from the four bitmap rows
// (r2 = r3 = nullptr for a CTA with one group): A at [0, nA), B at [nA, nA + nB),
// C after, each in increasing tile order, from a block-wide exclusive scan of
// the per-word class counts.  Rows of up to blockDim.x words take one pass;
// longer rows count first and write in a second pass.  When single-group tiles
// are rare (8 (nB + nC) < nA, the dynamic path's dense selections) the whole
// union is written as class A instead: both groups walk it in tile order.
// counts[0..2] = nA, nB, nC.  The caller's __syncthreads publishes the lists.
__device__ void build_fwd_lists(const uint32_t* r0, const uint32_t* r1, const uint32_t* r2,
                                const uint32_t* r3, int wq, uint16_t* list, int* counts,
                                int* scratch /* 3 * warps ints */) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const bool one_pass = wq <= (int)blockDim.x;
  int totA = 0, totB = 0;
  bool merged = false;
  for (int pass = one_pass ? 1 : 0; pass < 2; ++pass) {
    int baseA = 0, baseB = 0, baseC = 0;
    for (int w0 = 0; w0 < wq; w0 += blockDim.x) {
      const int w = w0 + tid;
      uint32_t g0 = 0, g1 = 0;
      if (w < wq) {
        g0 = __ldg(r0 + w) | __ldg(r1 + w);
        g1 = r2 != nullptr ? (__ldg(r2 + w) | __ldg(r3 + w)) : 0u;
      }
      uint32_t ca = g0 & g1, cb = g0 & ~g1, cc = g1 & ~g0;
      int xa = __popc(ca), xb = __popc(cb), xc = __popc(cc);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive warp scans
        const int ya = __shfl_up_sync(0xffffffffu, xa, o), yb = __shfl_up_sync(0xffffffffu, xb, o),
                  yc = __shfl_up_sync(0xffffffffu, xc, o);
        if (lane >= o) xa += ya, xb += yb, xc += yc;
      }
      if (lane == 31) scratch[3 * warp] = xa, scratch[3 * warp + 1] = xb, scratch[3 * warp + 2] = xc;
      __syncthreads();
      int ea = 0, eb = 0, ec = 0, ta = 0, tb = 0, tc = 0;
      for (int i = 0; i < nw; ++i) {
        const int sa = scratch[3 * i], sbb = scratch[3 * i + 1], scc = scratch[3 * i + 2];
        if (i < warp) ea += sa, eb += sbb, ec += scc;
        ta += sa, tb += sbb, tc += scc;
      }
      __syncthreads();
      if (one_pass) {  // the totals of the only chunk are the class sizes
        totA = ta, totB = tb;
        merged = 8 * (tb + tc) < ta;
      }
      if (pass == 1) {
        if (merged) {
          // union in tile order: class-A offsets plus the B and C entries before this word
          int o = baseA + baseB + baseC + ea + eb + ec + (xa - __popc(ca)) + (xb - __popc(cb)) +
                  (xc - __popc(cc));
          for (uint32_t m = g0 | g1; m; m &= m - 1u) list[o++] = (uint16_t)(w * 32 + __ffs(m) - 1);
        } else {
          int oa = baseA + ea + xa - __popc(ca);
          int ob = totA + baseB + eb + xb - __popc(cb);
          int oc = totA + totB + baseC + ec + xc - __popc(cc);
          for (uint32_t m = ca; m; m &= m - 1u) list[oa++] = (uint16_t)(w * 32 + __ffs(m) - 1);
          for (uint32_t m = cb; m; m &= m - 1u) list[ob++] = (uint16_t)(w * 32 + __ffs(m) - 1);
          for (uint32_t m = cc; m; m &= m - 1u) list[oc++] = (uint16_t)(w * 32 + __ffs(m) - 1);
        }
      }
      baseA += ta, baseB += tb, baseC += tc;
    }
    if (pass == 0) {
      totA = baseA;
      totB = baseB;
      merged = 8 * (baseB + baseC) < baseA;  // identical in every thread
    } else if (tid == 0) {
      if (merged) counts[0] = baseA + baseB + baseC, counts[1] = 0, counts[2] = 0;
      else counts[0] = baseA, counts[1] = baseB, counts[2] = baseC;
    }
  }
}

constexpr int kFwdThreads = 320;
constexpr int kFwdProducerWarp = 8;
constexpr int kFwdMmaWarp = 9;

// Design budget: shared-memory bandwidth (128 B/clk/SM), which the TMA fills,
// the tensor core's shared-memory operand reads and the mbarrier traffic all
// share, and the tcgen05.mma shape: an M = 128 product costs at least ~45
// clocks whatever its N, so N >= 128 is needed to run at the math rate.
// The forward therefore takes key tiles two at a time (S = Q [K_a; K_b]^T,
// N = 128), keeps P in TMEM (written by the softmax over the S columns it has
// read) as the A operand of P V, and shares each K/V pair between two groups
// of 128 query rows (256 rows per CTA), which halves the TMA bytes per FLOP.
template <int D>
struct FwdLayout {
  static constexpr int kRing = 2;                       // K pairs and V pairs in flight
  static constexpr int kSub = D / 64;                   // 128-byte sub-buffers per row
  static constexpr int kPair = kSub * 16384;            // one 128-row pair slot
  static constexpr int Q = 0;                           // 2 groups x 128 rows
  static constexpr int K = Q + 2 * kPair;               // kRing pair slots
  static constexpr int V = K + kRing * kPair;
  static constexpr int BAR = V + kRing * kPair;
  static constexpr int B_Q = 0, B_KF = 1, B_KE = B_KF + kRing, B_VF = B_KE + kRing,
                       B_VE = B_VF + kRing,
                       B_SF = B_VE + kRing,  // [g]: S_g ready
                       B_PF = B_SF + 2,      // [g]: P_g in TMEM (and O_g rescaled)
                       B_OF = B_PF + 2,      // [g]: last P V done
                       B_DRAIN = B_OF + 2, NBAR = B_DRAIN + 1;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr int COUNTS = ABORT + 4;           // 3 ints: class sizes
  static constexpr int SCRATCH = COUNTS + 16;        // 3 ints per warp (list build)
  static constexpr int LIST = SCRATCH + 3 * 4 * (kFwdThreads / 32);  // u16 per union tile
  // shared memory for n_tiles tiles (the class lists hold at most one entry per tile)
  static constexpr size_t bytes(int64_t n_tiles) { return 1024 + LIST + 2 * (size_t)n_tiles; }
  // TMEM per group g at 256 g: S (128 f32 columns; P as 64 bf16x2 columns over
  // its first half), O (D f32 columns)
  static constexpr int T_S = 0, T_O = 128;
};

// Per-key score offset (the kKeyBias form of the forward): S[r][c] += bias[64 t + c]
// for key tile t, in units of raw scores (a log-weight w becomes w / sm_scale).
template <bool kKeyBias>
__device__ __forceinline__ void add_key_bias(float (&s)[64], const float* __restrict__ key_bias,
                                             int t) {
  if constexpr (kKeyBias) {
    const float4* b4 = reinterpret_cast<const float4*>(key_bias + (int64_t)t * 64);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 b = __ldg(b4 + i);
      s[4 * i] += b.x;
      s[4 * i + 1] += b.y;
      s[4 * i + 2] += b.z;
      s[4 * i + 3] += b.w;
    }
  }
}

// Forward one-pass limit on a key tile's exponential sum (see the softmax loop).
constexpr float kFwdSumLimit = 65536.0f;

// Scores of keys outside the valid mask (bit c of vb clear) -> -inf.
__device__ __forceinline__ void mask_keys(float (&s)[64], uint64_t vb) {
#pragma unroll
  for (int c = 0; c < 64; ++c)
    if (!((vb >> c) & 1ull)) s[c] = -INFINITY;
}

__device__ __forceinline__ float tile_max(const float (&s)[64]) {
  float m0 = s[0], m1 = s[1], m2 = s[2], m3 = s[3];
#pragma unroll
  for (int c = 4; c < 64; c += 4) {
    m0 = fmaxf(m0, s[c]);
    m1 = fmaxf(m1, s[c + 1]);
    m2 = fmaxf(m2, s[c + 2]);
    m3 = fmaxf(m3, s[c + 3]);
  }
  return fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
}

// p = exp2(s * scale - m) for 64 scores as 32 bf16 pairs; returns the sum of the
// fp32 p (even and odd columns summed separately, then added).  The exponent
// arguments are packed f32x2 FFMAs (each lane rounds as fmaf does); the sums
// stay scalar (a packed accumulator costs registers the softmax does not have).
__device__ __forceinline__ float exp_tile(const float (&s)[64], float scale, float m, uint32_t (&pk)[32]) {
  const float2 sc = make_float2(scale, scale), nm = make_float2(-m, -m);
  float su0 = 0.f, su1 = 0.f;
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const float2 x = __ffma2_rn(make_float2(s[2 * c], s[2 * c + 1]), sc, nm);
    const float p0 = ex2(x.x), p1 = ex2(x.y);
    su0 += p0;
    su1 += p1;
    pk[c] = pack_bf16(p0, p1);
  }
  return su0 + su1;
}

// s[c] <- exp2(s[c] * scale + bias) for 64 scores (packed FFMA pairs).
__device__ __forceinline__ void exp_rows(float (&s)[64], float scale, float bias) {
  const float2 sc = make_float2(scale, scale), b = make_float2(bias, bias);
#pragma unroll
  for (int c = 0; c < 64; c += 2) {
    const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), sc, b);
    s[c] = ex2(x.x);
    s[c + 1] = ex2(x.y);
  }
}

// Rows of this warp's TMEM lanes, columns [0, 32 * NC) of taddr, times alpha.
template <int NC>
__device__ __forceinline__ void scale_tmem_rows(uint32_t taddr, float alpha) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    uint32_t raw[32];
    tmem_ld32(taddr + c * 32, raw);
    tmem_wait_ld_dep(raw);
#pragma unroll
    for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(u2f(raw[i]) * alpha);
    tmem_st32(taddr + c * 32, raw);
  }
}

// kKeyBias = false: the block-sparse forward (key validity tile_bits[key tile],
// shared by every query tile and head).  kKeyBias = true: the same kernel with a
// per-key score offset key_bias [Sk] and key masks per (head, query tile, key
// tile) at tile_bits[h * tb_hstride + q_tile * tb_qstride + key tile] (the
// pooled-key pass of the Taylor merge).
template <int D, bool kKeyBias = false>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, int64_t Sq, int64_t Sk, int wq, float qk_scale,
                  const uint32_t* __restrict__ bits_q, const uint64_t* __restrict__ tile_bits,
                  __nv_bfloat16* __restrict__ o, __nv_bfloat16* __restrict__ o_lo,
                  float* __restrict__ lse, const float* __restrict__ key_bias = nullptr,
                  int64_t tb_hstride = 0, int64_t tb_qstride = 0, int test_withhold = 0) {
  // test_withhold != 0 (prism_test_fwd_withheld_load only): the producer issues no
  // load at all, so the first wait of the MMA warp can only end at the wait limit
  using L = FwdLayout<D>;
  constexpr int R = L::kRing;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t sb = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = blockIdx.x, h = blockIdx.y;
  // queries: Sq rows per head (tiles in bits_q rows), keys: Sk rows per head; wq = words per
  // bits_q row (ceil(Sk / 2048))
  const int64_t n_tiles = Sq / 64;
  const bool g1_live = 4 * (int64_t)quad + 2 < n_tiles;  // Sq % 256 == 128: last CTA has one group
  const int row_base = (int)((int64_t)h * Sq + (int64_t)quad * 256);  // row of [heads*Sq, D]
  const int head_row = (int)((int64_t)h * Sk);                        // key rows of head h
  auto bar = [&](int i) { return sb + L::BAR + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::ABORT);
  const uint32_t* r0 = bits_q + ((int64_t)h * n_tiles + 4 * (int64_t)quad) * wq;
  const uint32_t* r2 = g1_live ? r0 + 2 * wq : nullptr;
  const uint32_t* r3 = g1_live ? r0 + 3 * wq : nullptr;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_Q), 1);
    for (int i = 0; i < R; ++i) {
      mbar_init(bar(L::B_KF + i), 1);
      mbar_init(bar(L::B_KE + i), 1);
      mbar_init(bar(L::B_VF + i), 1);
      mbar_init(bar(L::B_VE + i), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(L::B_SF + g), 1);
      mbar_init(bar(L::B_PF + g), 4);
      mbar_init(bar(L::B_OF + g), 1);
    }
    mbar_init(bar(L::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kFwdMmaWarp) {
    tmem_alloc(sb + L::TMEM_SLOT, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();  // barrier initialisation visible: the Q load overlaps the list build
  if (warp == kFwdProducerWarp && lane == 0 && !test_withhold) {
    const int nq = g1_live ? 4 : 2;  // 64-row Q blocks
    mbar_expect_tx(bar(L::B_Q), nq * 64 * D * 2);
    for (int qb = 0; qb < nq; ++qb)
#pragma unroll
      for (int s = 0; s < L::kSub; ++s)
        tma_load_2d(sb + L::Q + (qb >> 1) * L::kPair + s * 16384 + (qb & 1) * 8192, &tm_q, s * 64,
                    row_base + qb * 64, bar(L::B_Q));
  }
  uint16_t* list = reinterpret_cast<uint16_t*>(sm + L::LIST);
  build_fwd_lists(r0, r0 + wq, r2, r3, wq, list, reinterpret_cast<int*>(sm + L::COUNTS),
                  reinterpret_cast<int*>(sm + L::SCRATCH));
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + L::TMEM_SLOT);
  FwdSched sched;
  sched.init(list, reinterpret_cast<const int*>(sm + L::COUNTS));

  if (warp == kFwdProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !test_withhold) {
      int np = 0, t0, t1, mask;
      bool ok = true;
      for (int step = 0; step < sched.total; ++step) {
        sched.step(step, t0, t1, mask);
        const int cnt = t1 >= 0 ? 2 : 1;
        const int st = np % R;
        // K pair, then V pair, each into one 128-row slot (tile a rows 0-63, tile b 64-127)
        if (np >= R && !mbar_wait(bar(L::B_KE + st), ((np / R) - 1) & 1, abort_flag, &g_tc_error,
                                  kErrFwdProducer)) {
          ok = false;
          break;
        }
        mbar_expect_tx(bar(L::B_KF + st), cnt * 64 * D * 2);
        for (int u = 0; u < cnt; ++u)
#pragma unroll
          for (int s = 0; s < L::kSub; ++s)
            tma_load_2d(sb + L::K + st * L::kPair + s * 16384 + u * 8192, &tm_k, s * 64,
                        head_row + (u ? t1 : t0) * 64, bar(L::B_KF + st));
        if (np >= R && !mbar_wait(bar(L::B_VE + st), ((np / R) - 1) & 1, abort_flag, &g_tc_error,
                                  kErrFwdProducer)) {
          ok = false;
          ++np;  // the K pair of this step is in flight: drain it below
          break;
        }
        mbar_expect_tx(bar(L::B_VF + st), cnt * 64 * D * 2);
        for (int u = 0; u < cnt; ++u)
#pragma unroll
          for (int s = 0; s < L::kSub; ++s)
            tma_load_2d(sb + L::V + st * L::kPair + s * 16384 + u * 8192, &tm_v, s * 64,
                        head_row + (u ? t1 : t0) * 64, bar(L::B_VF + st));
        ++np;
      }
      // drain: every issued load has landed before the CTA may exit
      for (int m = (np > R ? np - R : 0); m < np; ++m) {
        mbar_wait(bar(L::B_KF + m % R), (m / R) & 1, abort_flag, &g_tc_error, kErrFwdProducer);
        if (ok || m + 1 < np)
          mbar_wait(bar(L::B_VF + m % R), (m / R) & 1, abort_flag, &g_tc_error, kErrFwdProducer);
      }
      mbar_wait(bar(L::B_Q), 0, abort_flag, &g_tc_error, kErrFwdProducer);
    }
  } else if (warp == kFwdMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    // Per step n, for the groups in its mask: PV_g(prev), S_g(n); then PV_g of
    // step n-1 for a group not in the mask.  S_g(n) overwrites the columns that
    // held P_g of the group's previous step, whose P V was issued at the step
    // after it (at the latest just before S_g(n)); the tensor pipe performs one
    // thread's MMAs in issue order.  Barrier parities count each group's steps.
    if (lane == 0) {
      constexpr uint32_t IDESC_S2 = idesc_bf16(128, 128, false, false);
      constexpr uint32_t IDESC_S1 = idesc_bf16(128, 64, false, false);
      constexpr uint32_t IDESC_PV = idesc_bf16(128, D, false, true);
      const int ng = g1_live ? 2 : 1;
      const uint64_t dQ = desc_k_sw128(sb + L::Q), dK = desc_k_sw128(sb + L::K),
                     dV = desc_mn_sw128(sb + L::V, 16384);
      bool ok = mbar_wait(bar(L::B_Q), 0, abort_flag, &g_tc_error, kErrFwdMma);
      tc_fence_after();
      // P V of group g's step j: K = 64 keys per tile of the pair, V in ring slot `slot`
      auto pv = [&](int g, int j, int cnt, int slot) -> bool {
        if (!mbar_wait(bar(L::B_PF + g), j & 1, abort_flag, &g_tc_error, kErrFwdMma)) return false;
        tc_fence_after();
        const uint64_t bv = dV + slot * (L::kPair >> 4);
        mma_ts_k64_mn(tmem + g * 256 + L::T_O, tmem + g * 256 + L::T_S, bv, IDESC_PV, j > 0 ? 1u : 0u);
        if (cnt == 2)
          mma_ts_k64_mn(tmem + g * 256 + L::T_O, tmem + g * 256 + L::T_S + 32, bv + (8192 >> 4),
                        IDESC_PV, 1u);
        return true;
      };
      int n = 0, prev_cnt = 0, prev_mask = 0, t0, t1, mask;
      int ns[2] = {0, 0};  // steps issued per group
      for (int step = 0; ok && step < sched.total; ++step) {
        sched.step(step, t0, t1, mask);
        if (!g1_live) mask &= 1;  // a CTA with one group: fallback steps are group 0's
        const int cnt = t1 >= 0 ? 2 : 1;
        const int st = n % R;
        if (!mbar_wait(bar(L::B_KF + st), (n / R) & 1, abort_flag, &g_tc_error, kErrFwdMma) ||
            (n > 0 && !mbar_wait(bar(L::B_VF + (n - 1) % R), ((n - 1) / R) & 1, abort_flag,
                                 &g_tc_error, kErrFwdMma))) {
          ok = false;
          break;
        }
        // groups of this step: P V of their previous step (its P occupies the
        // columns S is written to), then S; then P V for groups that sit this
        // step out, after the S products they need not wait for
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!((mask >> g) & 1)) continue;
          if (((prev_mask >> g) & 1) && !pv(g, ns[g] - 1, prev_cnt, (n - 1) % R)) {
            ok = false;
            break;
          }
          mma_kd<L::kSub, 16384, 16384>(tmem + g * 256 + L::T_S, dQ + g * (L::kPair >> 4),
                                        dK + st * (L::kPair >> 4),
                                        cnt == 2 ? IDESC_S2 : IDESC_S1, 0u);
          mma_commit(bar(L::B_SF + g));
          ++ns[g];
        }
        if (!ok) break;
#pragma unroll
        for (int g = 0; g < 2; ++g)
          if (((prev_mask >> g) & 1) && !((mask >> g) & 1) &&
              !pv(g, ns[g] - 1, prev_cnt, (n - 1) % R)) {
            ok = false;
            break;
          }
        if (!ok) break;
        mma_commit(bar(L::B_KE + st));
        if (n > 0) mma_commit(bar(L::B_VE + (n - 1) % R));
        prev_cnt = cnt;
        prev_mask = mask;
        ++n;
      }
      if (ok && n > 0) {
        if (mbar_wait(bar(L::B_VF + (n - 1) % R), ((n - 1) / R) & 1, abort_flag, &g_tc_error,
                      kErrFwdMma)) {
#pragma unroll
          for (int g = 0; g < 2; ++g)
            if (((prev_mask >> g) & 1) && !pv(g, ns[g] - 1, prev_cnt, (n - 1) % R)) {
              ok = false;
              break;
            }
          if (ok)
            for (int g = 0; g < ng; ++g)
              if (ns[g] > 0) mma_commit(bar(L::B_OF + g));
        }
      }
      // drain: all issued MMAs complete before TMEM is released
      mma_commit(bar(L::B_DRAIN));
      mbar_wait(bar(L::B_DRAIN), 0, abort_flag, &g_tc_error, kErrFwdMma);
    }
  } else if (warp < 4 || g1_live) {
    // ------------------------------------------------------ softmax warps
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // row within the group == TMEM lane
    const int sbit = 2 * g + (r >> 6);     // bitmap row of this thread's q tile
    const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16) + g * 256;
    float m = -INFINITY, l = 1.0f;
    const uint32_t* my_row = r0 + sbit * wq;  // this thread's q tile's bitmap row
    const uint64_t* tb = tile_bits;            // key masks of this thread's q tile
    if constexpr (kKeyBias) tb += (int64_t)h * tb_hstride + (4 * (int64_t)quad + sbit) * tb_qstride;
    int n = 0, t0, t1, mask;                   // n: this group's steps
    bool ok = true;
    for (int step = 0; step < sched.total; ++step) {
      sched.step(step, t0, t1, mask);
      if (!((mask >> g) & 1)) continue;
      const uint64_t vb0 = ((__ldg(my_row + (t0 >> 5)) >> (t0 & 31)) & 1u) ? tb[t0] : 0ull;
      const uint64_t vb1 =
          (t1 >= 0 && ((__ldg(my_row + (t1 >> 5)) >> (t1 & 31)) & 1u)) ? tb[t1] : 0ull;
      if (!warp_wait(bar(L::B_SF + g), n & 1, abort_flag, kErrFwdSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sum0 = 0.f, sum1 = 0.f;
      // Exponentials against the running maximum m in one pass over S.  A row's
      // first block (m = -inf) and a first key tile whose exponentials sum past
      // kFwdSumLimit (some p > 2^10, or an overflow) take two passes (maximum,
      // then exponentials: S is still intact then).  If only the second key tile
      // passes the limit, P of the first (already in TMEM) and l, O are scaled to
      // the new maximum and the second tile is recomputed from its scores
      // (columns [64, 128), intact).  Between rescales p <= 2^16, exact in fp32
      // and bf16's relative precision; the result is the same softmax in exact
      // arithmetic.  The one-pass path costs per score one packed FFMA, one ex2,
      // one packed FADD and half a bf16x2 conversion.
      bool two_pass = __any_sync(0xffffffffu, m == -INFINITY);
      uint32_t pk0[32];
      if (!two_pass) {
        if (vb0 == 0ull) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pk0[i] = 0u;
        } else {
          float sv[64];
          tmem_load<2>(t_lane + L::T_S, sv);
          add_key_bias<kKeyBias>(sv, key_bias, t0);
          if (vb0 != ~0ull) mask_keys(sv, vb0);
          sum0 = exp_tile(sv, qk_scale, m, pk0);
        }
        two_pass = __any_sync(0xffffffffu, !(sum0 <= kFwdSumLimit));
      }
      if (two_pass) {
        sum0 = 0.f;
        // pass 1: row maximum over the valid, selected keys (64 columns at a time)
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint64_t vb = u ? vb1 : vb0;
          if (vb == 0ull) continue;  // warp-uniform: the whole half-row of this tile is masked
          float s[64];
          tmem_load<2>(t_lane + L::T_S + u * 64, s);
          add_key_bias<kKeyBias>(s, key_bias, u ? t1 : t0);
          if (vb != ~0ull) mask_keys(s, vb);
          mx = fmaxf(mx, tile_max(s));
        }
        mx *= qk_scale;
        const bool need = mx > m + kRescaleThreshold;  // m = -inf: any valid key
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = need ? mx : m;
          const float alpha = need ? ex2(m - m_new) : 1.0f;  // m = -inf -> 0
          const bool o_live = __any_sync(0xffffffffu, need && m != -INFINITY);
          l *= alpha;
          m = m_new;
          // every P V before this pair has completed: S_g(n) was issued after them
          if (n > 0 && o_live) scale_tmem_rows<D / 32>(t_lane + L::T_O, alpha);
        }
        // pass 2: p = exp2(s * scale - m) -> bf16 P over the first 64 columns of S
        const float mb = (m == -INFINITY) ? 0.0f : m;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint64_t vb = u ? vb1 : vb0;
          uint32_t pk[32];
          if (vb == 0ull) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pk[i] = 0u;
          } else {
            float s[64];
            tmem_load<2>(t_lane + L::T_S + u * 64, s);
            add_key_bias<kKeyBias>(s, key_bias, u ? t1 : t0);
            if (vb != ~0ull) mask_keys(s, vb);
            const float t = exp_tile(s, qk_scale, mb, pk);
            if (u) sum1 = t; else sum0 = t;
          }
          // P columns [32 u, 32 u + 32) overlap S columns [0, 64), which pass 2
          // has already read for u = 0 and does not read again
          tmem_st32(t_lane + L::T_S + u * 32, pk);
        }
      } else {
        // P columns [0, 32) overlap S columns [0, 64) of the first key tile (read)
        tmem_st32(t_lane + L::T_S, pk0);
        uint32_t pk1[32];
        if (vb1 == 0ull) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pk1[i] = 0u;
        } else {
          float sv[64];
          tmem_load<2>(t_lane + L::T_S + 64, sv);
          add_key_bias<kKeyBias>(sv, key_bias, t1);
          if (vb1 != ~0ull) mask_keys(sv, vb1);
          sum1 = exp_tile(sv, qk_scale, m, pk1);
        }
        const bool need = !(sum1 <= kFwdSumLimit);
        if (__any_sync(0xffffffffu, need)) {
          // rare: rescale to this row's new maximum (tile 1's scores, columns
          // [64, 128) of S, are still intact in TMEM)
          float sv[64];
          tmem_load<2>(t_lane + L::T_S + 64, sv);
          add_key_bias<kKeyBias>(sv, key_bias, t1);
          if (vb1 != ~0ull) mask_keys(sv, vb1);
          {
            const float m_new = need ? fmaxf(m, tile_max(sv) * qk_scale) : m;
            const float alpha = ex2(m - m_new);
            if (n > 0) scale_tmem_rows<D / 32>(t_lane + L::T_O, alpha);
            tmem_wait_st();
            {
              uint32_t raw[32];
              tmem_ld32(t_lane + L::T_S, raw);
              tmem_wait_ld_dep(raw);
#pragma unroll
              for (int i = 0; i < 32; ++i)
                raw[i] = pack_bf16(u2f(raw[i] << 16) * alpha, u2f(raw[i] & 0xffff0000u) * alpha);
              tmem_st32(t_lane + L::T_S, raw);
            }
            l = (l + sum0) * alpha;
            sum0 = 0.f;
            m = m_new;
            sum1 = exp_tile(sv, qk_scale, m, pk1);
          }
        }
        // P columns [32, 64) overlap S columns [32, 64) of the first key tile (read)
        tmem_st32(t_lane + L::T_S + 32, pk1);
      }
      l += sum0 + sum1;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_PF + g));
      ++n;
    }
    // epilogue
    const int64_t grow = (int64_t)row_base + g * 128 + r;
    if (ok && n > 0 && warp_wait(bar(L::B_OF + g), 0, abort_flag, kErrFwdSoftmax)) {
      tc_fence_after();
      const float inv = 1.0f / l;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t raw[32];
        tmem_ld32(t_lane + L::T_O + c * 32, raw);
        tmem_wait_ld_dep(raw);
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = u2f(raw[2 * i]) * inv, x1 = u2f(raw[2 * i + 1]) * inv;
          hi[i] = pack_bf16(x0, x1);
          lo[i] = pack_bf16(x0 - u2f(hi[i] << 16), x1 - u2f(hi[i] & 0xffff0000u));
        }
        uint4* dst = reinterpret_cast<uint4*>(o + grow * D + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
        if (o_lo != nullptr) {
          uint4* dl = reinterpret_cast<uint4*>(o_lo + grow * D + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dl[i] = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
        }
      }
      lse[grow] = (m + __log2f(l)) * kLn2;
    } else if (ok && n == 0) {
      // no selected tile at all: O = 0, lse = -inf (m = -inf, l = 1)
      uint4* dst = reinterpret_cast<uint4*>(o + grow * D);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
      if (o_lo != nullptr) {
        uint4* dl = reinterpret_cast<uint4*>(o_lo + grow * D);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dl[i] = make_uint4(0, 0, 0, 0);
      }
      lse[grow] = -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kFwdMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------ dK / dV softmax (both kernels)
// The transposed softmax reads the 16x256b TMEM layout.  A softmax warp covers
// its 32 key lanes x the 64 query columns of one tile.  With 16x256b loads a
// thread holds, in each 16-lane half, key lanes a and a + 8 (a = lane / 4) at
// the column pairs 8 j + 2 (lane % 4) + {0, 1}, j = 0..7: 16 query columns
// rather than a whole row's 64, so it reads 16 lse and 16 delta values per tile
// (one 8-byte load per column pair; a warp's load touches 4 addresses: one
// shared-memory wavefront).  A thread owning a whole key row would need all 64
// values of both, broadcast by 16-byte loads at 4 wavefronts each -- half of
// the shared-memory port at the tensor core's rate, which the MMA operand reads
// and TMA fills need.  The bf16 pairs go back with 16x128b stores, whose
// layout puts packed column 4 j + lane % 4 of lanes a, a + 8 in the registers
// that hold them.
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Key validity of this thread's four lanes: bit 2 hl + kk <=> key lane
// 32 q + 16 hl + 8 kk + lane / 4 of the CTA is valid (q = lane quarter of the warp).
__device__ __forceinline__ uint32_t dkdv_lane_valid(uint64_t tile_valid_bits, int quarter, int lane) {
  uint32_t v = 0;
#pragma unroll
  for (int hl = 0; hl < 2; ++hl)
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int row = 32 * quarter + 16 * hl + 8 * kk + (lane >> 2);
      v |= (uint32_t)((tile_valid_bits >> (row & 63)) & 1ull) << (2 * hl + kk);
    }
  return v;
}

// P^T of one query tile for this warp: p[32 hl + 4 j + 2 kk + e] = exp2(s * scale -
// lse[col] / ln 2) (0 for an invalid key lane or an unselected tile), written as bf16
// pairs over the first 32 of the tile's 64 S^T columns.  t_tile = TMEM address of
// the warp's lane quarter at the tile's first S^T column.
__device__ __forceinline__ void dkdv_p_tile(uint32_t t_tile, const float* __restrict__ lse_t,
                                            float qk_scale, bool tile_on, uint32_t lane_valid,
                                            int lane, float (&p)[64]) {
  const int c2 = 2 * (lane & 3);
  const float2 sc = make_float2(qk_scale, qk_scale), nr = make_float2(-kRcpLn2, -kRcpLn2);
#pragma unroll
  for (int hl = 0; hl < 2; ++hl) {
    uint32_t pk[16];
    if (tile_on) {
      uint32_t raw[32];
      tmem_ld_16x256b_x8(t_tile + ((uint32_t)(16 * hl) << 16), raw);
      tmem_wait_ld_dep(raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // -(lse * c) == lse * (-c) exactly; each lane of the packed ops rounds as fmaf / fmul
        const float2 nl = __fmul2_rn(*reinterpret_cast<const float2*>(lse_t + 8 * j + c2), nr);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const bool on = (lane_valid >> (2 * hl + kk)) & 1u;
          const float2 x = __ffma2_rn(make_float2(u2f(raw[4 * j + 2 * kk]), u2f(raw[4 * j + 2 * kk + 1])), sc, nl);
          const float e0 = on ? ex2(x.x) : 0.0f, e1 = on ? ex2(x.y) : 0.0f;
          p[32 * hl + 4 * j + 2 * kk] = e0;
          p[32 * hl + 4 * j + 2 * kk + 1] = e1;
          pk[2 * j + kk] = pack_bf16(e0, e1);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) p[32 * hl + i] = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = 0u;
    }
    // bf16 columns [0, 32) of the tile over S^T columns this half has read
    tmem_st_16x128b_x8(t_tile + ((uint32_t)(16 * hl) << 16), pk);
  }
}

// dS^T = P^T (dP^T - delta[col]) of one query tile as bf16 pairs over the first 32
// of the tile's 64 dP^T columns (t_tile: the warp's lane quarter at the tile's first
// dP^T column).
__device__ __forceinline__ void dkdv_ds_tile(uint32_t t_tile, const float* __restrict__ delta_t,
                                             bool tile_on, int lane, const float (&p)[64]) {
  const int c2 = 2 * (lane & 3);
  const float2 neg1 = make_float2(-1.0f, -1.0f);
#pragma unroll
  for (int hl = 0; hl < 2; ++hl) {
    uint32_t pk[16];
    if (tile_on) {
      uint32_t raw[32];
      tmem_ld_16x256b_x8(t_tile + ((uint32_t)(16 * hl) << 16), raw);
      tmem_wait_ld_dep(raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 d2 = *reinterpret_cast<const float2*>(delta_t + 8 * j + c2);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int i = 32 * hl + 4 * j + 2 * kk;
          // dp - delta as fma(delta, -1, dp): the same single rounding as the subtraction
          const float2 ds = __fmul2_rn(make_float2(p[i], p[i + 1]),
                                       __ffma2_rn(d2, neg1, make_float2(u2f(raw[4 * j + 2 * kk]),
                                                                        u2f(raw[4 * j + 2 * kk + 1]))));
          pk[2 * j + kk] = pack_bf16(ds.x, ds.y);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = 0u;
    }
    tmem_st_16x128b_x8(t_tile + ((uint32_t)(16 * hl) << 16), pk);
  }
}

// ============================================================= dK / dV, N = 128
// CTA = 128 keys (tiles 2p, 2p+1); per step TWO query tiles of the transposed
// selection's union (N = 128; the last step holds one tile when the union is
// odd).  TMEM: dK, dV (D f32 columns each), S^T and dP^T (128 f32 columns
// each, single-buffered): S^T = K Q^T, dP^T = V dO^T; warpgroup w (w = query
// tile w of the step) writes P^T and dS^T = P^T (dP^T - delta) as bf16 over
// its own 64 columns [64 w, 64 w + 32) of them; dV += P^T dO and dK += dS^T Q
// read them from TMEM.  Per step the tensor pipe runs S^T, dP^T, dV, dK with
// N >= 128 (the math rate), and the issuer synchronises once per two query
// tiles instead of once per tile.
template <int D>
struct Dkdv2Layout {
  static constexpr int kRing = 2;                          // query-tile pairs in flight
  static constexpr int kSub = D / 64;
  static constexpr int kPair = kSub * 16384;               // 128 rows (two tiles) x D bf16
  static constexpr int K = 0;                              // 128 keys
  static constexpr int V = K + kPair;
  static constexpr int Q = V + kPair;                      // kRing pairs of query tiles
  static constexpr int DO = Q + kRing * kPair;
  static constexpr int M = DO + kRing * kPair;             // kRing x 128 f32 (lse)
  static constexpr int DL = M + kRing * 512;               // kRing x 128 f32 (delta)
  static constexpr int BAR = DL + kRing * 512;
  static constexpr int B_KV = 0, B_QF = 1, B_QE = 1 + kRing, B_SF = 1 + 2 * kRing,
                       B_DPF = B_SF + 1, B_PF = B_DPF + 1, B_DSF = B_PF + 1, B_FIN = B_DSF + 1,
                       B_DRAIN = B_FIN + 1, NBAR = B_DRAIN + 1;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr size_t kBytes = 1024 + ABORT + 4;
  static constexpr int T_DK = 0, T_DV = D, T_S = 2 * D, T_DP = 2 * D + 128;
  static_assert(T_DP + 128 <= 512, "TMEM budget");
};

// Pairs of consecutive union tiles: (t0, sel0, t1, sel1), t1 = -1 for a lone last tile.
struct UnionPairIter {
  UnionIter it;
  __device__ __forceinline__ void init(const uint32_t* ra, const uint32_t* rb, int wq) {
    it.init(ra, rb, wq);
  }
  __device__ __forceinline__ bool next(int& t0, int& s0, int& t1, int& s1) {
    t0 = it.next(s0);
    if (t0 < 0) return false;
    t1 = it.next(s1);
    if (t1 < 0) s1 = 0;
    return true;
  }
};

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    dkdv2_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const float* __restrict__ lse, const float* __restrict__ delta, int64_t Sq,
                    int64_t Sk, int wq, float qk_scale, float sm_scale,
                    const uint32_t* __restrict__ bits_k, const uint64_t* __restrict__ tile_bits,
                    __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv) {
  using L = Dkdv2Layout<D>;
  constexpr int R = L::kRing;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t sb = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x, h = blockIdx.y;
  const int64_t n_tiles = Sk / 64;
  const int row_base = (int)((int64_t)h * Sk + (int64_t)pair * 128);  // key rows of this CTA
  const int head_row = (int)((int64_t)h * Sq);                        // query rows of head h
  auto bar = [&](int i) { return sb + L::BAR + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::ABORT);
  const uint32_t* row_a = bits_k + ((int64_t)h * n_tiles + 2 * (int64_t)pair) * wq;
  const uint32_t* row_b = row_a + wq;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_KV), 1);
    for (int i = 0; i < R; ++i) {
      mbar_init(bar(L::B_QF + i), 1);
      mbar_init(bar(L::B_QE + i), 1);
    }
    mbar_init(bar(L::B_SF), 1);
    mbar_init(bar(L::B_DPF), 1);
    mbar_init(bar(L::B_PF), 8);
    mbar_init(bar(L::B_DSF), 8);
    mbar_init(bar(L::B_FIN), 1);
    mbar_init(bar(L::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kBwdMmaWarp) {
    tmem_alloc(sb + L::TMEM_SLOT, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + L::TMEM_SLOT);

  if (warp == kBwdProducerWarp) {
    if (lane == 0) {
      mbar_expect_tx(bar(L::B_KV), 2 * 128 * D * 2);
#pragma unroll
      for (int s = 0; s < L::kSub; ++s)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          tma_load_2d(sb + L::K + s * 16384 + r * 8192, &tm_k, s * 64, row_base + r * 64, bar(L::B_KV));
          tma_load_2d(sb + L::V + s * 16384 + r * 8192, &tm_v, s * 64, row_base + r * 64, bar(L::B_KV));
        }
      UnionPairIter it;
      it.init(row_a, row_b, wq);
      int n = 0, t0, s0, t1, s1;
      while (it.next(t0, s0, t1, s1)) {
        const int st = n & 1, cnt = t1 >= 0 ? 2 : 1;
        if (n >= R && !mbar_wait(bar(L::B_QE + st), ((n >> 1) - 1) & 1, abort_flag, &g_tc_error,
                                 kErrDkdvProducer))
          break;
        mbar_expect_tx(bar(L::B_QF + st), cnt * (2 * 64 * D * 2 + 2 * 256));
        for (int u = 0; u < cnt; ++u) {
          const int t = u ? t1 : t0;
#pragma unroll
          for (int s = 0; s < L::kSub; ++s) {
            tma_load_2d(sb + L::Q + st * L::kPair + s * 16384 + u * 8192, &tm_q, s * 64,
                        head_row + t * 64, bar(L::B_QF + st));
            tma_load_2d(sb + L::DO + st * L::kPair + s * 16384 + u * 8192, &tm_do, s * 64,
                        head_row + t * 64, bar(L::B_QF + st));
          }
          bulk_load(sb + L::M + st * 512 + u * 256, lse + head_row + (int64_t)t * 64, 256,
                    bar(L::B_QF + st));
          bulk_load(sb + L::DL + st * 512 + u * 256, delta + head_row + (int64_t)t * 64, 256,
                    bar(L::B_QF + st));
        }
        ++n;
      }
      for (int m = (n > R ? n - R : 0); m < n; ++m)
        mbar_wait(bar(L::B_QF + (m & 1)), (m >> 1) & 1, abort_flag, &g_tc_error, kErrDkdvProducer);
      mbar_wait(bar(L::B_KV), 0, abort_flag, &g_tc_error, kErrDkdvProducer);
    }
  } else if (warp == kBwdMmaWarp) {
    // Issue order: S^T(n) | dK(n-1) | dP^T(n) | dV(n), ... , dK(last).
    // The softmax computes P^T(n) while the tensor pipe runs dK(n-1) and dP^T(n),
    // and dS^T(n) while it runs dV(n) and S^T(n+1).  S^T(n) overwrites P^T(n-1),
    // read by dV(n-1); dP^T(n) overwrites dS^T(n-1), read by dK(n-1): both readers
    // are issued earlier, and one thread's MMAs run in issue order.
    if (lane == 0) {
      constexpr uint32_t IDESC_S2 = idesc_bf16(128, 128, false, false);
      constexpr uint32_t IDESC_S1 = idesc_bf16(128, 64, false, false);
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);
      const uint64_t dK = desc_k_sw128(sb + L::K), dV = desc_k_sw128(sb + L::V),
                     dQk = desc_k_sw128(sb + L::Q), dDOk = desc_k_sw128(sb + L::DO),
                     dQmn = desc_mn_sw128(sb + L::Q, 16384), dDOmn = desc_mn_sw128(sb + L::DO, 16384);
      constexpr uint32_t kSlot = L::kPair >> 4;  // descriptor step of one ring slot
      const int tiles = union_count(row_a, row_b, wq);
      const int steps = (tiles + 1) >> 1;
      // dK += dS^T Q for step j (slot j & 1), after its dS^T is written
      auto dk_step = [&](int j) -> bool {
        const uint32_t js = (uint32_t)j & 1u;
        if (!mbar_wait(bar(L::B_DSF), js, abort_flag, &g_tc_error, kErrDkdvMma)) return false;
        tc_fence_after();
        mma_ts_chain4<8, 16, 24, 128, 256, 384>(tmem + L::T_DK, tmem + L::T_DP, dQmn + js * kSlot,
                                                IDESC_G, j > 0 ? 1u : 0u);
        if (2 * j + 1 < tiles)
          mma_ts_chain4<8, 16, 24, 128, 256, 384>(tmem + L::T_DK, tmem + L::T_DP + 64,
                                                  dQmn + js * kSlot + 512, IDESC_G, 1u);
        mma_commit(bar(L::B_QE + js));
        return true;
      };
      bool ok = mbar_wait(bar(L::B_KV), 0, abort_flag, &g_tc_error, kErrDkdvMma);
      tc_fence_after();
      for (int n = 0; ok && n < steps; ++n) {
        const uint32_t st = (uint32_t)n & 1u, ph = (uint32_t)n & 1u;
        const bool two = 2 * n + 1 < tiles;
        const uint32_t idn = two ? IDESC_S2 : IDESC_S1;
        if (!mbar_wait(bar(L::B_QF + st), ((uint32_t)n >> 1) & 1u, abort_flag, &g_tc_error,
                       kErrDkdvMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        mma_kd<L::kSub, 16384, 16384>(tmem + L::T_S, dK, dQk + st * kSlot, idn, 0u);
        mma_commit(bar(L::B_SF));
        if (n > 0 && !dk_step(n - 1)) {
          ok = false;
          break;
        }
        mma_kd<L::kSub, 16384, 16384>(tmem + L::T_DP, dV, dDOk + st * kSlot, idn, 0u);
        mma_commit(bar(L::B_DPF));
        if (!mbar_wait(bar(L::B_PF), ph, abort_flag, &g_tc_error, kErrDkdvMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // K = query rows: tile 0's P^T in columns [0, 32), tile 1's in [64, 96)
        mma_ts_chain4<8, 16, 24, 128, 256, 384>(tmem + L::T_DV, tmem + L::T_S, dDOmn + st * kSlot,
                                                IDESC_G, n > 0 ? 1u : 0u);
        if (two)
          mma_ts_chain4<8, 16, 24, 128, 256, 384>(tmem + L::T_DV, tmem + L::T_S + 64,
                                                  dDOmn + st * kSlot + 512, IDESC_G, 1u);
      }
      if (ok && steps > 0) dk_step(steps - 1);
      mma_commit(bar(L::B_FIN));
      mma_commit(bar(L::B_DRAIN));
      mbar_wait(bar(L::B_DRAIN), 0, abort_flag, &g_tc_error, kErrDkdvMma);
    }
  } else {
    // softmax warpgroups: wg w takes query tile w of each step (64 columns)
    const int wg = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // key row of the epilogue == TMEM lane
    const int half = (warp & 3) >> 1;      // this warp's key tile of the CTA
    const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t lane_valid = dkdv_lane_valid(tile_bits[2 * pair + half], warp & 3, lane);
    UnionPairIter it;
    it.init(row_a, row_b, wq);
    int n = 0, t0, s0, t1, s1;
    bool ok = true;
    const float* sM = reinterpret_cast<const float*>(sm + L::M);
    const float* sDl = reinterpret_cast<const float*>(sm + L::DL);
    while (it.next(t0, s0, t1, s1)) {
      const int st = n & 1, ph = n & 1;
      const int sel = wg ? s1 : s0;
      const bool tile_on = (wg == 0 || t1 >= 0) && ((sel >> half) & 1);  // warp-uniform
      if (!warp_wait(bar(L::B_QF + st), (n >> 1) & 1, abort_flag, kErrDkdvSoftmax) ||
          !warp_wait(bar(L::B_SF), ph, abort_flag, kErrDkdvSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tcol = wg * 64;
      float p[64];
      dkdv_p_tile(t_lane + L::T_S + tcol, sM + st * 128 + wg * 64, qk_scale, tile_on, lane_valid, lane, p);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_PF));
      if (!warp_wait(bar(L::B_DPF), ph, abort_flag, kErrDkdvSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      dkdv_ds_tile(t_lane + L::T_DP + tcol, sDl + st * 128 + wg * 64, tile_on, lane, p);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_DSF));
      ++n;
    }
    // epilogue: wg 0 writes dK (scaled by sm_scale), wg 1 writes dV
    const int64_t grow = (int64_t)row_base + r;
    __nv_bfloat16* out = (wg == 0 ? dk : dv) + grow * D;
    const float scale = wg == 0 ? sm_scale : 1.0f;
    const int tcolo = wg == 0 ? L::T_DK : L::T_DV;
    if (ok && n > 0 && warp_wait(bar(L::B_FIN), 0, abort_flag, kErrDkdvSoftmax)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t raw[32], pk2[16];
        tmem_ld32(t_lane + tcolo + c * 32, raw);
        tmem_wait_ld_dep(raw);
#pragma unroll
        for (int i = 0; i < 16; ++i) pk2[i] = pack_bf16(u2f(raw[2 * i]) * scale, u2f(raw[2 * i + 1]) * scale);
        uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk2[4 * i], pk2[4 * i + 1], pk2[4 * i + 2], pk2[4 * i + 3]);
      }
    } else if (ok && n == 0) {
      uint4* a = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) a[i] = make_uint4(0, 0, 0, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kBwdMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ======================================================================= dQ
// CTA = 128 queries (tiles 2p, 2p+1); per step a PAIR of key tiles (N = 128):
// S = Q [K_a; K_b]^T and dP = dO [V_a; V_b]^T in TMEM; the softmax warpgroups
// (wg 0: key tile a, wg 1: key tile b) compute dS = P (dP - delta) into TMEM
// columns of its own, and dQ += dS [K_a; K_b] reads them from there.  The MMA
// thread issues S(n+1) and dP(n+1) as soon as the softmax has read S(n) and
// dP(n), and dQ(n) when dS(n) is written, so the tensor core works on the next
// pair while the softmax of this one runs.
template <int D>
struct DqLayout {
  static constexpr int kRingK = 3;                         // K pairs (used by S and dQ)
  static constexpr int kRingV = 2;                         // V pairs (used by dP)
  static constexpr int kSub = D / 64;
  static constexpr int kPair = kSub * 16384;
  static constexpr int Q = 0;                              // 128 queries
  static constexpr int DO = Q + kPair;
  static constexpr int K = DO + kPair;
  static constexpr int V = K + kRingK * kPair;
  static constexpr int BAR = V + kRingV * kPair;
  static constexpr int B_QD = 0, B_KF = 1, B_KE = B_KF + kRingK, B_VF = B_KE + kRingK,
                       B_VE = B_VF + kRingV, B_SF = B_VE + kRingV, B_DPF = B_SF + 1,
                       B_DPE = B_DPF + 1, B_DSF = B_DPE + 1, B_DSE = B_DSF + 1, B_FIN = B_DSE + 1,
                       B_DRAIN = B_FIN + 1, NBAR = B_DRAIN + 1;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr size_t kBytes = 1024 + ABORT + 4;
  // TMEM: dQ (D f32 columns), S and dP (128 f32 columns each), dS (key tile u
  // as 32 bf16x2 columns at T_DS + 32 u)
  static constexpr int T_DQ = 0, T_S = 128, T_DP = 256, T_DS = 384;
};

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    dq_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                 const float* __restrict__ lse, const float* __restrict__ delta, int64_t Sq, int64_t Sk,
                 int wq, float qk_scale, float sm_scale, const uint32_t* __restrict__ bits_q,
                 const uint64_t* __restrict__ tile_bits, __nv_bfloat16* __restrict__ dq) {
  using L = DqLayout<D>;
  constexpr int RK = L::kRingK, RV = L::kRingV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t sb = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x, h = blockIdx.y;
  // queries: tile pair `pair` of Sq rows per head (rows of bits_q); keys: Sk rows per head,
  // wq = words per bits_q row (ceil(Sk / 2048))
  const int64_t n_tiles = Sq / 64;
  const int row_base = (int)((int64_t)h * Sq + (int64_t)pair * 128);  // query rows of this CTA
  const int head_row = (int)((int64_t)h * Sk);                        // key rows of head h
  auto bar = [&](int i) { return sb + L::BAR + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::ABORT);
  const uint32_t* row_a = bits_q + ((int64_t)h * n_tiles + 2 * (int64_t)pair) * wq;
  const uint32_t* row_b = row_a + wq;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_QD), 1);
    for (int i = 0; i < RK; ++i) {
      mbar_init(bar(L::B_KF + i), 1);
      mbar_init(bar(L::B_KE + i), 1);
    }
    for (int i = 0; i < RV; ++i) {
      mbar_init(bar(L::B_VF + i), 1);
      mbar_init(bar(L::B_VE + i), 1);
    }
    mbar_init(bar(L::B_SF), 1);
    mbar_init(bar(L::B_DPF), 1);
    mbar_init(bar(L::B_DPE), 8);
    mbar_init(bar(L::B_DSF), 8);
    mbar_init(bar(L::B_DSE), 1);
    mbar_init(bar(L::B_FIN), 1);
    mbar_init(bar(L::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kBwdMmaWarp) {
    tmem_alloc(sb + L::TMEM_SLOT, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + L::TMEM_SLOT);

  if (warp == kBwdProducerWarp) {
    if (lane == 0) {
      mbar_expect_tx(bar(L::B_QD), 2 * 128 * D * 2);
#pragma unroll
      for (int s = 0; s < L::kSub; ++s)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          tma_load_2d(sb + L::Q + s * 16384 + r * 8192, &tm_q, s * 64, row_base + r * 64, bar(L::B_QD));
          tma_load_2d(sb + L::DO + s * 16384 + r * 8192, &tm_do, s * 64, row_base + r * 64, bar(L::B_QD));
        }
      UnionIter it;
      it.init(row_a, row_b, wq);
      int nk = 0, nv = 0, sel = 0;
      for (;;) {
        const int t0 = it.next(sel);
        if (t0 < 0) break;
        const int t1 = it.next(sel);
        const int cnt = t1 >= 0 ? 2 : 1;
        const int sk = nk % RK, sv = nv % RV;
        if (nk >= RK && !mbar_wait(bar(L::B_KE + sk), ((nk / RK) - 1) & 1, abort_flag, &g_tc_error,
                                   kErrDqProducer))
          break;
        mbar_expect_tx(bar(L::B_KF + sk), cnt * 64 * D * 2);
        for (int u = 0; u < cnt; ++u)
#pragma unroll
          for (int s = 0; s < L::kSub; ++s)
            tma_load_2d(sb + L::K + sk * L::kPair + s * 16384 + u * 8192, &tm_k, s * 64,
                        head_row + (u ? t1 : t0) * 64, bar(L::B_KF + sk));
        ++nk;
        if (nv >= RV && !mbar_wait(bar(L::B_VE + sv), ((nv / RV) - 1) & 1, abort_flag, &g_tc_error,
                                   kErrDqProducer))
          break;
        mbar_expect_tx(bar(L::B_VF + sv), cnt * 64 * D * 2);
        for (int u = 0; u < cnt; ++u)
#pragma unroll
          for (int s = 0; s < L::kSub; ++s)
            tma_load_2d(sb + L::V + sv * L::kPair + s * 16384 + u * 8192, &tm_v, s * 64,
                        head_row + (u ? t1 : t0) * 64, bar(L::B_VF + sv));
        ++nv;
        if (t1 < 0) break;
      }
      for (int m = (nk > RK ? nk - RK : 0); m < nk; ++m)
        mbar_wait(bar(L::B_KF + m % RK), (m / RK) & 1, abort_flag, &g_tc_error, kErrDqProducer);
      for (int m = (nv > RV ? nv - RV : 0); m < nv; ++m)
        mbar_wait(bar(L::B_VF + m % RV), (m / RV) & 1, abort_flag, &g_tc_error, kErrDqProducer);
      mbar_wait(bar(L::B_QD), 0, abort_flag, &g_tc_error, kErrDqProducer);
    }
  } else if (warp == kBwdMmaWarp) {
    // Issue order: S(0) dP(0) | S(1) dP(1) dQ(0) | S(2) dP(2) dQ(1) | ...
    // S(n+1) and dP(n+1) wait until the softmax has read S(n) and dP(n) (one
    // signal, B_DPE: it reads dP after S), dQ(n) until dS(n) is written.  The
    // issuing thread keeps its loop minimal -- the tensor pipe's issue queue is
    // shallow, so every instruction and wait between MMAs is time the pipe may
    // idle: a counted loop (the tile sequence itself is not needed here) with
    // the ring slots advanced incrementally.
    if (lane == 0) {
      constexpr uint32_t IDESC_2 = idesc_bf16(128, 128, false, false);
      constexpr uint32_t IDESC_1 = idesc_bf16(128, 64, false, false);
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);
      const uint64_t dQ = desc_k_sw128(sb + L::Q), dDO = desc_k_sw128(sb + L::DO),
                     dKk = desc_k_sw128(sb + L::K), dVk = desc_k_sw128(sb + L::V),
                     dKmn = desc_mn_sw128(sb + L::K, 16384);
      static_assert(RV == 2, "V ring arithmetic below assumes 2 slots");
      constexpr uint32_t kSlot = L::kPair >> 4;  // descriptor step of one ring slot
      const int tiles = union_count(row_a, row_b, wq);
      const int steps = (tiles + 1) >> 1;
      bool ok = mbar_wait(bar(L::B_QD), 0, abort_flag, &g_tc_error, kErrDqMma);
      tc_fence_after();
      // dQ += dS K for step j (K pair in ring slot `slot`)
      auto dq_step = [&](int j, uint32_t slot, bool two) -> bool {
        if (!mbar_wait(bar(L::B_DSF), (uint32_t)j & 1u, abort_flag, &g_tc_error, kErrDqMma)) return false;
        tc_fence_after();
        const uint64_t bk = dKmn + slot * kSlot;
        mma_ts_k64_mn(tmem + L::T_DQ, tmem + L::T_DS, bk, IDESC_G, j > 0 ? 1u : 0u);
        if (two) mma_ts_k64_mn(tmem + L::T_DQ, tmem + L::T_DS + 32, bk + (8192 >> 4), IDESC_G, 1u);
        mma_commit(bar(L::B_DSE));
        mma_commit(bar(L::B_KE + slot));
        return true;
      };
      uint32_t sk = 0, kpar = 0, psk = 0;  // K slot / phase of step n, K slot of step n - 1
      for (int n = 0; ok && n < steps; ++n) {
        const bool two = 2 * n + 1 < tiles;
        const uint32_t idn = two ? IDESC_2 : IDESC_1, sv = (uint32_t)n & 1u;
        if (!mbar_wait(bar(L::B_KF + sk), kpar, abort_flag, &g_tc_error, kErrDqMma) ||
            (n > 0 && !mbar_wait(bar(L::B_DPE), (uint32_t)(n - 1) & 1u, abort_flag, &g_tc_error,
                                 kErrDqMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        mma_kd<L::kSub, 16384, 16384>(tmem + L::T_S, dQ, dKk + sk * kSlot, idn, 0u);
        mma_commit(bar(L::B_SF));
        if (!mbar_wait(bar(L::B_VF + sv), ((uint32_t)n >> 1) & 1u, abort_flag, &g_tc_error,
                       kErrDqMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        mma_kd<L::kSub, 16384, 16384>(tmem + L::T_DP, dDO, dVk + sv * kSlot, idn, 0u);
        mma_commit(bar(L::B_DPF));
        mma_commit(bar(L::B_VE + sv));
        if (n > 0 && !dq_step(n - 1, psk, true)) {  // only the last step can be a single tile
          ok = false;
          break;
        }
        psk = sk;
        if (++sk == (uint32_t)RK) {
          sk = 0;
          kpar ^= 1u;
        }
      }
      if (ok && steps > 0) dq_step(steps - 1, psk, 2 * (steps - 1) + 1 < tiles);
      mma_commit(bar(L::B_FIN));
      mma_commit(bar(L::B_DRAIN));
      mbar_wait(bar(L::B_DRAIN), 0, abort_flag, &g_tc_error, kErrDqMma);
    }
  } else {
    // softmax warpgroups: wg 0 takes key tile a of each pair, wg 1 tile b
    const int wg = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // query row within the CTA == TMEM lane
    const int half = r >> 6;
    const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int64_t grow = (int64_t)row_base + r;
    const float mrow = lse[grow] * kRcpLn2;
    const float drow = delta[grow];
    UnionIter it;
    it.init(row_a, row_b, wq);
    int n = 0, sel0 = 0, sel1 = 0;
    bool ok = true;
    for (;;) {
      const int t0 = it.next(sel0);
      if (t0 < 0) break;
      const int t1 = it.next(sel1);
      const bool live = wg == 0 || t1 >= 0;  // warp-uniform
      const int tw = wg == 0 ? t0 : t1;
      const int selw = wg == 0 ? sel0 : sel1;
      const uint64_t vb = (live && ((selw >> half) & 1)) ? tile_bits[tw] : 0ull;  // warp-uniform
      if (!warp_wait(bar(L::B_SF), n & 1, abort_flag, kErrDqSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S(n) and dP(n) are both read into registers before the exponentials and
      // released at once (B_DPE), so the tensor core computes S(n+1) and dP(n+1)
      // while this step's exp2 (1,024 MUFU clocks per step for the SM) and dS run.
      // dS(n) overwrites dS(n-1): its stores wait until dQ(n-1) has read it
      // (B_DSE); it is written in two halves of 16 columns to bound registers.
      float p[64], dp[64];
      if (vb != 0ull) tmem_load<2>(t_lane + L::T_S + wg * 64, p);
      if (!warp_wait(bar(L::B_DPF), n & 1, abort_flag, kErrDqSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (vb != 0ull) tmem_load<2>(t_lane + L::T_DP + wg * 64, dp);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_DPE));
      if (vb != 0ull && vb != ~0ull) mask_keys(p, vb);  // masked keys: exp2(-inf) = 0
      const float2 sc = make_float2(qk_scale, qk_scale), nm = make_float2(-mrow, -mrow),
                   nd = make_float2(-drow, -drow);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t pk[16];
        if (vb != 0ull) {
#pragma unroll
          for (int c = 32 * hh; c < 32 * hh + 32; c += 2) {
            const float2 x = __ffma2_rn(make_float2(p[c], p[c + 1]), sc, nm);
            const float2 ds = __fmul2_rn(make_float2(ex2(x.x), ex2(x.y)),
                                         __fadd2_rn(make_float2(dp[c], dp[c + 1]), nd));
            pk[(c - 32 * hh) / 2] = pack_bf16(ds.x, ds.y);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = 0u;
        }
        if (hh == 0) {
          if (n > 0 && !warp_wait(bar(L::B_DSE), (n - 1) & 1, abort_flag, kErrDqSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (live) tmem_st16(t_lane + L::T_DS + wg * 32 + 16 * hh, pk);
      }
      if (!ok) break;
      if (live) tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_DSF));
      ++n;
      if (t1 < 0) break;
    }
    // epilogue: wg 0 writes dQ columns [0, D/2), wg 1 [D/2, D)
    if (ok && n > 0 && warp_wait(bar(L::B_FIN), 0, abort_flag, kErrDqSoftmax)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        const int col = wg * (D / 2) + c * 32;
        uint32_t raw[32], pk[16];
        tmem_ld32(t_lane + L::T_DQ + col, raw);
        tmem_wait_ld_dep(raw);
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(u2f(raw[2 * i]) * sm_scale, u2f(raw[2 * i + 1]) * sm_scale);
        uint4* dst = reinterpret_cast<uint4*>(dq + grow * D + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    } else if (ok && n == 0) {
      uint4* a = reinterpret_cast<uint4*>(dq + grow * D + wg * (D / 2));
#pragma unroll
      for (int i = 0; i < D / 16; ++i) a[i] = make_uint4(0, 0, 0, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kBwdMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================ preprocess
// delta[h][s] = sum_d O * dO (fp32), one warp per row; with o_lo (the
// forward's rounding residual) the row uses O = hi + lo.
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

// ================================================================ host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// [rows, D] bf16 row-major, 64 x 64 boxes, 128-byte swizzle.
static prism_status_t make_map(CUtensorMap* map, const void* ptr, int64_t rows, int D, const char* what) {
  EncodeFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable from the driver", what);
    return PRISM_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
    return PRISM_ERR_CUDA;
  }
  return PRISM_OK;
}

#define PRISM_TRY(x)                       \
  do {                                     \
    prism_status_t st_ = (x);              \
    if (st_ != PRISM_OK) return st_;       \
  } while (0)

template <int D, bool kKeyBias = false>
prism_status_t launch_fwd(const void* q, const void* k, const void* v, int heads, int64_t Sq,
                          int64_t Sk, float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                          void* o, void* o_lo, float* lse, cudaStream_t stream,
                          const float* key_bias = nullptr, int64_t tb_hstride = 0,
                          int64_t tb_qstride = 0, int test_withhold = 0) {
  const int64_t n_tiles = Sq / 64, n_ktiles = Sk / 64;
  const int wq = (int)((n_ktiles + 31) / 32);
  const size_t need = FwdLayout<D>::bytes(n_ktiles);
  const size_t sm = need > kMinSmem ? need : kMinSmem;
  PRISM_CHECK_ARG(n_ktiles <= 65536 && sm <= 227 * 1024,
                  "prism_bsa_fwd: %lld key tiles per head exceed the shared-memory tile lists",
                  (long long)n_ktiles);
  CUtensorMap mq, mk, mv;
  PRISM_TRY(make_map(&mq, q, (int64_t)heads * Sq, D, "prism_bsa_fwd"));
  PRISM_TRY(make_map(&mk, k, (int64_t)heads * Sk, D, "prism_bsa_fwd"));
  PRISM_TRY(make_map(&mv, v, (int64_t)heads * Sk, D, "prism_bsa_fwd"));
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(fwd_tc_kernel<D, kKeyBias>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_fwd: smem attribute");
  fwd_tc_kernel<D, kKeyBias><<<dim3((unsigned)((n_tiles + 3) / 4), heads), kFwdThreads, sm, stream>>>(
      mq, mk, mv, Sq, Sk, wq, sm_scale * kRcpLn2, bits_q, tile_bits, (__nv_bfloat16*)o,
      (__nv_bfloat16*)o_lo, lse, key_bias, tb_hstride, tb_qstride, test_withhold);
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
prism_status_t launch_dkdv2(const void* q, const void* k, const void* v, const void* dout,
                            const float* lse, const float* delta, int heads, int64_t Sq, int64_t Sk,
                            float sm_scale, const uint32_t* bits_k, const uint64_t* tile_bits,
                            void* dk, void* dv, cudaStream_t stream) {
  const int64_t n_ktiles = Sk / 64;
  const int wq = (int)((Sq / 64 + 31) / 32);  // words per bits_k row (query tiles)
  const size_t sm = Dkdv2Layout<D>::kBytes > kMinSmem ? Dkdv2Layout<D>::kBytes : kMinSmem;
  PRISM_CHECK_ARG(sm <= 227 * 1024, "prism_bsa_bwd: shared memory layout exceeds 227 KB");
  CUtensorMap mq, mk, mv, mdo;
  PRISM_TRY(make_map(&mq, q, (int64_t)heads * Sq, D, "prism_bsa_bwd_dkdv"));
  PRISM_TRY(make_map(&mk, k, (int64_t)heads * Sk, D, "prism_bsa_bwd_dkdv"));
  PRISM_TRY(make_map(&mv, v, (int64_t)heads * Sk, D, "prism_bsa_bwd_dkdv"));
  PRISM_TRY(make_map(&mdo, dout, (int64_t)heads * Sq, D, "prism_bsa_bwd_dkdv"));
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(dkdv2_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_bwd: smem attribute");
  dkdv2_tc_kernel<D><<<dim3((unsigned)(n_ktiles / 2), heads), kBwdThreads, sm, stream>>>(
      mq, mk, mv, mdo, lse, delta, Sq, Sk, wq, sm_scale * kRcpLn2, sm_scale, bits_k, tile_bits,
      (__nv_bfloat16*)dk, (__nv_bfloat16*)dv);
  PRISM_CHECK_LAUNCH("prism_bsa_bwd_dkdv");
  return PRISM_OK;
}

template <int D>
prism_status_t launch_dq(const void* q, const void* k, const void* v, const void* dout,
                         const float* lse, const float* delta, int heads, int64_t Sq, int64_t Sk,
                         float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                         void* dq, cudaStream_t stream) {
  const int64_t n_tiles = Sq / 64;
  const int wq = (int)((Sk / 64 + 31) / 32);  // words per bits_q row (key tiles)
  const size_t sm = DqLayout<D>::kBytes > kMinSmem ? DqLayout<D>::kBytes : kMinSmem;
  PRISM_CHECK_ARG(sm <= 227 * 1024, "prism_bsa_bwd: shared memory layout exceeds 227 KB");
  CUtensorMap mq, mk, mv, mdo;
  PRISM_TRY(make_map(&mq, q, (int64_t)heads * Sq, D, "prism_bsa_bwd_dq"));
  PRISM_TRY(make_map(&mk, k, (int64_t)heads * Sk, D, "prism_bsa_bwd_dq"));
  PRISM_TRY(make_map(&mv, v, (int64_t)heads * Sk, D, "prism_bsa_bwd_dq"));
  PRISM_TRY(make_map(&mdo, dout, (int64_t)heads * Sq, D, "prism_bsa_bwd_dq"));
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(dq_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                   "prism_bsa_bwd: smem attribute");
  dq_tc_kernel<D><<<dim3((unsigned)(n_tiles / 2), heads), kBwdThreads, sm, stream>>>(
      mq, mk, mv, mdo, lse, delta, Sq, Sk, wq, sm_scale * kRcpLn2, sm_scale, bits_q, tile_bits,
      (__nv_bfloat16*)dq);
  PRISM_CHECK_LAUNCH("prism_bsa_bwd_dq");
  return PRISM_OK;
}

}  // namespace tc
}  // namespace prism

using namespace prism;

int prism_gemm_device_status_internal(void);

extern "C" {

int prism_device_status(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_tc_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(tc::g_tc_error, &zero, sizeof(int));
  }
  const int g = prism_gemm_device_status_internal();  // the GEMM kernels' word (gemm_tc.cu)
  if (g < 0) return -1;
  return v != 0 ? v : g;
}

// Row indices of the [heads * S, D] views are 32-bit TMA coordinates.
#define PRISM_ATTN_LEN_CHECKS(name, S)                                                            \
  PRISM_CHECK_ARG(S > 0 && S % 128 == 0 && heads >= 1,                                            \
                  name ": sequence lengths must be positive multiples of 128");                   \
  PRISM_CHECK_ARG((int64_t)heads * S < ((int64_t)1 << 31), name ": heads * S must be below 2^31")
#define PRISM_ATTN_SHAPE_CHECKS(name, Sq, Sk)                                                     \
  PRISM_ATTN_LEN_CHECKS(name, Sq);                                                                \
  PRISM_ATTN_LEN_CHECKS(name, Sk);                                                                \
  PRISM_CHECK_ARG(D == 64 || D == 128, name ": head dim %d not supported (64, 128)", D)

prism_status_t prism_bsa_fwd_qk(const void* q, const void* k, const void* v, int heads, int64_t Sq,
                                int64_t Sk, int D, float sm_scale, const uint32_t* bits_q,
                                const uint64_t* tile_bits, void* o, void* o_lo, float* lse,
                                cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && bits_q && tile_bits && o && lse, "prism_bsa_fwd: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_bsa_fwd", Sq, Sk);
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o), "prism_bsa_fwd: tensors must be 16-byte aligned");
  PRISM_CHECK_ARG(o_lo == nullptr || aligned16(o_lo), "prism_bsa_fwd: o_lo must be 16-byte aligned");
  if (D == 128) return tc::launch_fwd<128>(q, k, v, heads, Sq, Sk, sm_scale, bits_q, tile_bits, o, o_lo, lse, stream);
  return tc::launch_fwd<64>(q, k, v, heads, Sq, Sk, sm_scale, bits_q, tile_bits, o, o_lo, lse, stream);
}

prism_status_t prism_bsa_fwd_keybias(const void* q, const void* k, const void* v, int heads, int64_t Sq,
                                     int64_t Sk, int D, float sm_scale, const uint32_t* bits_q,
                                     const uint64_t* key_masks, const float* key_bias, void* o,
                                     void* o_lo, float* lse, cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && bits_q && key_masks && key_bias && o && lse,
                  "prism_bsa_fwd_keybias: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_bsa_fwd_keybias", Sq, Sk);
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) && aligned16(key_bias),
                  "prism_bsa_fwd_keybias: tensors must be 16-byte aligned");
  PRISM_CHECK_ARG(o_lo == nullptr || aligned16(o_lo), "prism_bsa_fwd_keybias: o_lo must be 16-byte aligned");
  const int64_t n_qt = Sq / 64, n_kt = Sk / 64;
  if (D == 128)
    return tc::launch_fwd<128, true>(q, k, v, heads, Sq, Sk, sm_scale, bits_q, key_masks, o, o_lo, lse,
                                     stream, key_bias, n_qt * n_kt, n_kt);
  return tc::launch_fwd<64, true>(q, k, v, heads, Sq, Sk, sm_scale, bits_q, key_masks, o, o_lo, lse,
                                  stream, key_bias, n_qt * n_kt, n_kt);
}

prism_status_t prism_bsa_fwd(const void* q, const void* k, const void* v, int heads, int64_t S,
                             int D, float sm_scale, const uint32_t* bits_q,
                             const uint64_t* tile_bits, void* o, void* o_lo, float* lse,
                             cudaStream_t stream) {
  return prism_bsa_fwd_qk(q, k, v, heads, S, S, D, sm_scale, bits_q, tile_bits, o, o_lo, lse, stream);
}

prism_status_t prism_test_fwd_withheld_load(const void* q, const void* k, const void* v, int64_t S,
                                            int D, float sm_scale, const uint32_t* bits_q,
                                            const uint64_t* tile_bits, void* o, float* lse,
                                            uint64_t wait_limit_ns, cudaStream_t stream) {
  const int heads = 1;
  PRISM_CHECK_ARG(q && k && v && bits_q && tile_bits && o && lse, "prism_test_fwd_withheld_load: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_test_fwd_withheld_load", S, S);
  PRISM_CHECK_ARG(S <= 256, "prism_test_fwd_withheld_load: S must be at most 256 (one CTA)");
  PRISM_CHECK_ARG(wait_limit_ns >= 100000ull && wait_limit_ns <= tc::kDefaultWaitLimitNs,
                  "prism_test_fwd_withheld_load: wait limit must be in [0.1 ms, 2 s]");
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o),
                  "prism_test_fwd_withheld_load: tensors must be 16-byte aligned");
  // stream-ordered: the shortened limit is in place for this launch only
  static const unsigned long long kDefault = tc::kDefaultWaitLimitNs;
  static thread_local unsigned long long limit;
  limit = (unsigned long long)wait_limit_ns;
  PRISM_CHECK_CUDA(cudaMemcpyToSymbolAsync(tc::g_wait_limit_ns, &limit, sizeof(limit), 0,
                                           cudaMemcpyHostToDevice, stream),
                   "prism_test_fwd_withheld_load: set wait limit");
  const prism_status_t st =
      D == 128 ? tc::launch_fwd<128>(q, k, v, heads, S, S, sm_scale, bits_q, tile_bits, o, nullptr, lse,
                                     stream, nullptr, 0, 0, 1)
               : tc::launch_fwd<64>(q, k, v, heads, S, S, sm_scale, bits_q, tile_bits, o, nullptr, lse,
                                    stream, nullptr, 0, 0, 1);
  PRISM_CHECK_CUDA(cudaMemcpyToSymbolAsync(tc::g_wait_limit_ns, &kDefault, sizeof(kDefault), 0,
                                           cudaMemcpyHostToDevice, stream),
                   "prism_test_fwd_withheld_load: restore wait limit");
  PRISM_CHECK_CUDA(cudaStreamSynchronize(stream), "prism_test_fwd_withheld_load: synchronize");
  return st;
}

size_t prism_bsa_bwd_workspace_bytes(int heads, int64_t S) {
  return (size_t)heads * (size_t)S * sizeof(float);
}

prism_status_t prism_bsa_bwd_delta(const void* o, const void* o_lo, const void* dout, int heads,
                                   int64_t S, int D, float* delta, cudaStream_t stream) {
  PRISM_CHECK_ARG(o && dout && delta, "prism_bsa_bwd_delta: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_bsa_bwd_delta", S, S);
  return D == 128 ? tc::launch_delta<128>(o, o_lo, dout, heads, S, delta, stream)
                  : tc::launch_delta<64>(o, o_lo, dout, heads, S, delta, stream);
}

static prism_status_t bwd_dkdv_qk(const void* q, const void* k, const void* v, const void* dout,
                                  const float* lse, const float* delta, int heads, int64_t Sq,
                                  int64_t Sk, int D, float sm_scale, const uint32_t* bits_k,
                                  const uint64_t* tile_bits, void* dk, void* dv, cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && dout && lse && delta && bits_k && tile_bits && dk && dv,
                  "prism_bsa_bwd_dkdv: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_bsa_bwd_dkdv", Sq, Sk);
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dout) && aligned16(dk) &&
                      aligned16(dv) && aligned16(lse) && aligned16(delta),
                  "prism_bsa_bwd_dkdv: tensors must be 16-byte aligned");
  return D == 128 ? tc::launch_dkdv2<128>(q, k, v, dout, lse, delta, heads, Sq, Sk, sm_scale, bits_k, tile_bits, dk, dv, stream)
                  : tc::launch_dkdv2<64>(q, k, v, dout, lse, delta, heads, Sq, Sk, sm_scale, bits_k, tile_bits, dk, dv, stream);
}

static prism_status_t bwd_dq_qk(const void* q, const void* k, const void* v, const void* dout,
                                const float* lse, const float* delta, int heads, int64_t Sq,
                                int64_t Sk, int D, float sm_scale, const uint32_t* bits_q,
                                const uint64_t* tile_bits, void* dq, cudaStream_t stream) {
  PRISM_CHECK_ARG(q && k && v && dout && lse && delta && bits_q && tile_bits && dq, "prism_bsa_bwd_dq: null pointer");
  PRISM_ATTN_SHAPE_CHECKS("prism_bsa_bwd_dq", Sq, Sk);
  PRISM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dout) && aligned16(dq),
                  "prism_bsa_bwd_dq: tensors must be 16-byte aligned");
  return D == 128 ? tc::launch_dq<128>(q, k, v, dout, lse, delta, heads, Sq, Sk, sm_scale, bits_q, tile_bits, dq, stream)
                  : tc::launch_dq<64>(q, k, v, dout, lse, delta, heads, Sq, Sk, sm_scale, bits_q, tile_bits, dq, stream);
}

prism_status_t prism_bsa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout,
                                  const float* lse, const float* delta, int heads, int64_t S, int D,
                                  float sm_scale, const uint32_t* bits_k, const uint64_t* tile_bits,
                                  void* dk, void* dv, cudaStream_t stream) {
  return bwd_dkdv_qk(q, k, v, dout, lse, delta, heads, S, S, D, sm_scale, bits_k, tile_bits, dk, dv, stream);
}

prism_status_t prism_bsa_bwd_dq(const void* q, const void* k, const void* v, const void* dout,
                                const float* lse, const float* delta, int heads, int64_t S, int D,
                                float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                                void* dq, cudaStream_t stream) {
  return bwd_dq_qk(q, k, v, dout, lse, delta, heads, S, S, D, sm_scale, bits_q, tile_bits, dq, stream);
}

prism_status_t prism_bsa_bwd_qk(const void* q, const void* k, const void* v, const void* o,
                                const void* o_lo, const void* dout, const float* lse, int heads,
                                int64_t Sq, int64_t Sk, int D, float sm_scale,
                                const uint32_t* bits_q, const uint32_t* bits_k,
                                const uint64_t* tile_bits, void* workspace, void* dq, void* dk,
                                void* dv, cudaStream_t stream) {
  PRISM_CHECK_ARG(workspace, "prism_bsa_bwd: null pointer");
  float* delta = (float*)workspace;
  prism_status_t st = prism_bsa_bwd_delta(o, o_lo, dout, heads, Sq, D, delta, stream);
  if (st != PRISM_OK) return st;
  st = bwd_dkdv_qk(q, k, v, dout, lse, delta, heads, Sq, Sk, D, sm_scale, bits_k, tile_bits, dk, dv, stream);
  if (st != PRISM_OK) return st;
  return bwd_dq_qk(q, k, v, dout, lse, delta, heads, Sq, Sk, D, sm_scale, bits_q, tile_bits, dq, stream);
}

prism_status_t prism_bsa_bwd(const void* q, const void* k, const void* v, const void* o,
                             const void* o_lo, const void* dout, const float* lse, int heads,
                             int64_t S, int D,
                             float sm_scale, const uint32_t* bits_q, const uint32_t* bits_k,
                             const uint64_t* tile_bits, void* workspace, void* dq, void* dk,
                             void* dv, cudaStream_t stream) {
  return prism_bsa_bwd_qk(q, k, v, o, o_lo, dout, lse, heads, S, S, D, sm_scale, bits_q, bits_k,
                          tile_bits, workspace, dq, dk, dv, stream);
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
// the first call made on that device (again if the current context changed).
namespace prism {
namespace tc {
static __device__ __align__(256) float g_noalloc_delta[PRISM_BSA_BWD_NOALLOC_MAX_ROWS];
}  // namespace tc

static std::mutex g_noalloc_mu;
// Per device: the context the address was looked up under, and the address.
struct NoallocSlot {
  CUcontext ctx;
  float* addr;
};
static NoallocSlot g_noalloc_slot[128] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
static CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

static prism_status_t noalloc_scratch(float** out) {
  int dev = -1;
  PRISM_CHECK_CUDA(cudaGetDevice(&dev), "prism_bsa_bwd_noalloc: cudaGetDevice");
  PRISM_CHECK_ARG(dev >= 0 && dev < 128, "prism_bsa_bwd_noalloc: device ordinal %d out of range", dev);
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  PRISM_CHECK_ARG(get_ctx != nullptr, "prism_bsa_bwd_noalloc: cuCtxGetCurrent is unavailable from the driver");
  // A host thread may not have a current context yet; the runtime call below
  // makes the device's primary context current, so the context is read again.
  CUcontext ctx = nullptr;
  PRISM_CHECK_ARG(get_ctx(&ctx) == CUDA_SUCCESS, "prism_bsa_bwd_noalloc: cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc_slot[dev];
  if (slot.addr == nullptr || ctx == nullptr || slot.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, tc::g_noalloc_delta);
    if (e != cudaSuccess || p == nullptr) {
      set_error("prism_bsa_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return PRISM_ERR_CUDA;
    }
    PRISM_CHECK_ARG(get_ctx(&ctx) == CUDA_SUCCESS && ctx != nullptr,
                    "prism_bsa_bwd_noalloc: no current CUDA context");
    slot.ctx = ctx;
    slot.addr = static_cast<float*>(p);
  }
  *out = slot.addr;
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
