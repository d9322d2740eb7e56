// PREP kernels: the LSSA-B8 quantisers (P1 query rows, P2 K/V 128-key blocks, P3 the B9.1
// sink value grid).  Memory-bound byte work: one warp per query row, one CTA per
// (batch, kv head, key block).  Max reductions are exact and order-free, so warp shuffles
// are used freely; nothing here rounds except rint(x * 2^e), which is exact-or-zero.
#pragma once
#include "common.cuh"

namespace lssab8 {

struct Strides4 { long long s0, s1, s2, s3; };

// P1 (reference/t10_attn.py:40-48; golden reference/lssab_golden.py:228-229).
// x [B, H, T, dh] (any strides) -> q8 [B, H, Tpad, dh] int8, eq [B, H, Tpad] int32.
// Rows t in [T, Tpad) are written as zeros (they are padding for the 128-row TMA tiles).
template <typename InT>
__global__ void __launch_bounds__(256)
quant_rows_kernel(const InT* __restrict__ x, Strides4 xs, int B, int H, int T, int dh, int Tpad,
                  int8_t* __restrict__ q8, int32_t* __restrict__ eq) {
  const int warps = blockDim.x >> 5;
  const long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long nrows = (long long)B * H * Tpad;
  if (row >= nrows) return;
  const int t = (int)(row % Tpad);
  const long long bh = row / Tpad;
  const int h = (int)(bh % H), b = (int)(bh / H);
  int8_t* dst = q8 + row * dh;
  if (t >= T) {
    for (int c = lane; c < dh; c += 32) dst[c] = 0;
    if (lane == 0) eq[row] = 0;
    return;
  }
  const InT* src = x + b * xs.s0 + h * xs.s1 + (long long)t * xs.s2;
  constexpr int kMaxPer = 8;                  // dh <= 256
  float v[kMaxPer];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int c = lane + 32 * i;
    v[i] = (c < dh) ? to_f32(src[(long long)c * xs.s3]) : 0.0f;
    m = fmaxf(m, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int e = pow2_exponent(m, 40);
  const float sc = pow2f(e);
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int c = lane + 32 * i;
    if (c < dh) dst[c] = (int8_t)quant8(v[i], sc);
  }
  if (lane == 0) eq[row] = e;
}

// P1 with one exponent per head (q_exp_mode "head", reference/lssab_golden.py:230-232): the same
// rule over all T rows and dh channels of a head.  One CTA per (head, batch): pass 1 the head's
// amax, pass 2 every row on that exponent; eq[b, h, t] = e_h for t < T.  Rows [T, Tpad) zero.
template <typename InT>
__global__ void __launch_bounds__(256)
quant_head_kernel(const InT* __restrict__ x, Strides4 xs, int B, int H, int T, int dh, int Tpad,
                  int8_t* __restrict__ q8, int32_t* __restrict__ eq) {
  __shared__ float red[8];
  const int h = blockIdx.x, b = blockIdx.y;
  const InT* src = x + b * xs.s0 + h * xs.s1;
  const long long n = (long long)T * dh;
  float m = 0.0f;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    const long long t = i / dh, c = i % dh;
    m = fmaxf(m, fabsf(to_f32(src[t * xs.s2 + c * xs.s3])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  const int e = pow2_exponent(m, 40);
  const float sc = pow2f(e);
  const long long row0 = ((long long)b * H + h) * Tpad;
  int8_t* dst = q8 + row0 * dh;
  for (long long i = threadIdx.x; i < (long long)Tpad * dh; i += blockDim.x) {
    const long long t = i / dh, c = i % dh;
    dst[i] = t < T ? (int8_t)quant8(to_f32(src[t * xs.s2 + c * xs.s3]), sc) : (int8_t)0;
  }
  for (int t = threadIdx.x; t < Tpad; t += blockDim.x) eq[row0 + t] = t < T ? e : 0;
}

// B9.3 value quantiser (v_keyshift = dmax, reference/lssab9_golden.py:37-70; reference/
// lssab9_torch.py:145-153).  One CTA per (key block, kv head, batch).  The block exponent e_v is
// the B9 value grid's (modes 1 / 2 of quant_blocks_kernel: clamp [-32, 48], then outside [-32, 40]
// sets kDevEvRange; mode 2 quantises key 0 alone, e0, when T > 1).  Key j then sits on the grid
// e_tok + d_j, e_tok = e_v (e0 for key 0 in mode 2), d_j = clamp(e_j - e_tok, 0, dmax) with e_j the
// key's own exponent on the B9 grid (its row alone); x8 = clamp(rint(x 2^(e_tok + d_j)), +-127)
// and d8[b, g, j] = d_j (padding keys 0).  One warp per key row in pass 2.
template <typename InT>
__global__ void __launch_bounds__(256)
quant_values_keyshift_kernel(const InT* __restrict__ x, Strides4 xs, int B, int KVH, int T, int dh, int Tpad,
                             int mode, int dmax, int8_t* __restrict__ x8, int32_t* __restrict__ eblk,
                             int32_t* __restrict__ e0, int8_t* __restrict__ d8, int* __restrict__ err) {
  const int blk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int nblk = (T + kKB - 1) / kKB;
  const int lo = blk * kKB;
  const int hi = min(T, lo + kKB);
  const InT* src = x + b * xs.s0 + g * xs.s1;
  const long long rowbase = (long long)(b * KVH + g) * Tpad;
  int8_t* dst = x8 + rowbase * dh;
  const bool split0 = (mode == 2) && (blk == 0) && (T > 1);
  __shared__ float red[2][8];
  float m = 0.0f, m0 = 0.0f;
  const int n = (hi - lo) * dh;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = lo + i / dh, c = i % dh;
    const float a = fabsf(to_f32(src[(long long)r * xs.s2 + (long long)c * xs.s3]));
    if (split0 && r == 0) m0 = fmaxf(m0, a); else m = fmaxf(m, a);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
  }
  if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = m; red[1][threadIdx.x >> 5] = m0; }
  __syncthreads();
  m = 0.0f; m0 = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { m = fmaxf(m, red[0][w]); m0 = fmaxf(m0, red[1][w]); }
  const int e = pow2_exponent(m, 48);
  const int ez = split0 ? pow2_exponent(m0, 48) : e;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = lo + warp; r < hi; r += (int)(blockDim.x >> 5)) {      // one warp per key row
    const InT* xr = src + (long long)r * xs.s2;
    float mr = 0.0f;
    for (int c = lane; c < dh; c += 32) mr = fmaxf(mr, fabsf(to_f32(xr[(long long)c * xs.s3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, o));
    const int etok = (split0 && r == 0) ? ez : e;
    const int dj = min(max(pow2_exponent(mr, 48) - etok, 0), dmax);
    const float sc = pow2f(etok + dj);
    for (int c = lane; c < dh; c += 32) dst[(long long)r * dh + c] = (int8_t)quant8(to_f32(xr[(long long)c * xs.s3]), sc);
    if (lane == 0) d8[rowbase + r] = (int8_t)dj;
  }
  if (blk == nblk - 1) {                             // padding rows of the last block
    for (int i = threadIdx.x; i < (Tpad - hi) * dh; i += blockDim.x) dst[(long long)hi * dh + i] = 0;
    for (int r = hi + threadIdx.x; r < Tpad; r += blockDim.x) d8[rowbase + r] = 0;
  }
  if (threadIdx.x == 0) {
    eblk[(long long)(b * KVH + g) * nblk + blk] = e;
    if (mode == 2 && blk == 0) e0[b * KVH + g] = ez;
    if (e < -32 || e > 40) atomicOr(err, kDevEvRange);
  }
}

// P2/P3 (reference/lssab_torch.py:62-85; reference/lssab9_torch.py:46-65,121-132,158).
// One CTA per (key block, kv head, batch).  x [B, KVH, T, dh] -> x8 [B, KVH, Tpad, dh],
// e [B, KVH, nblk], e0 [B, KVH] (sink mode only).
//   mode 0: B8 grid, exponent clamp [-32, 40]
//   mode 1: B9 value grid, clamp [-32, 48], then e outside [-32, 40] sets kDevEvRange
//   mode 2: B9.1 sink_alone: as mode 1, and when T > 1 key 0 is quantised alone (e0) while
//           block 0's exponent covers keys 1 .. min(KB, T)-1.
// mu [KVH, dh] (keys only, may be null): the key offset, subtracted in binary32 before both
// passes, k' = fl(f32(k) - mu[g, c]) (reference/lssab_golden.py:221, reference/lssab8_torch.py:143-144).
template <typename InT>
__global__ void __launch_bounds__(256)
quant_blocks_kernel(const InT* __restrict__ x, Strides4 xs, int B, int KVH, int T, int dh, int Tpad,
                    int mode, int8_t* __restrict__ x8, int32_t* __restrict__ eblk, int32_t* __restrict__ e0,
                    const float* __restrict__ mu, int* __restrict__ err) {
  const int blk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int nblk = (T + kKB - 1) / kKB;
  const int lo = blk * kKB;
  const int hi = min(T, lo + kKB);
  const InT* src = x + b * xs.s0 + g * xs.s1;
  int8_t* dst = x8 + ((long long)(b * KVH + g) * Tpad) * dh;
  const bool split0 = (mode == 2) && (blk == 0) && (T > 1);
  __shared__ float red[2][8];
  // pass 1: amax over the block's present rows (and key 0 alone when split0)
  float m = 0.0f, m0 = 0.0f;
  const int n = (hi - lo) * dh;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int r = lo + i / dh, c = i % dh;
    float a = to_f32(src[(long long)r * xs.s2 + (long long)c * xs.s3]);
    if (mu) a = __fsub_rn(a, mu[g * dh + c]);
    a = fabsf(a);
    if (split0 && r == 0) m0 = fmaxf(m0, a); else m = fmaxf(m, a);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
  }
  if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = m; red[1][threadIdx.x >> 5] = m0; }
  __syncthreads();
  m = 0.0f; m0 = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { m = fmaxf(m, red[0][w]); m0 = fmaxf(m0, red[1][w]); }
  const int hic = (mode == 0) ? 40 : 48;
  const int e = pow2_exponent(m, hic);
  const int ez = split0 ? pow2_exponent(m0, 48) : e;
  const float sc = pow2f(e), sc0 = pow2f(ez);
  // pass 2: quantise (re-reading the block keeps registers free; it is L2/L1 resident)
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int r = lo + i / dh, c = i % dh;
    float v = to_f32(src[(long long)r * xs.s2 + (long long)c * xs.s3]);
    if (mu) v = __fsub_rn(v, mu[g * dh + c]);
    dst[(long long)r * dh + c] = (int8_t)quant8(v, (split0 && r == 0) ? sc0 : sc);
  }
  // zero the padding rows of the last block
  if (blk == nblk - 1) {
    const int npad = (Tpad - hi) * dh;
    for (int i = threadIdx.x; i < npad; i += blockDim.x) dst[(long long)hi * dh + i] = 0;
  }
  if (threadIdx.x == 0) {
    eblk[(long long)(b * KVH + g) * nblk + blk] = e;
    if (mode == 2 && blk == 0) e0[b * KVH + g] = ez;
    if (mode != 0 && (e < -32 || e > 40)) atomicOr(err, kDevEvRange);
  }
}

// ------------------------------------------------------------ vectorised fast paths
// Used when the channel dimension is contiguous and every row starts on a 16-byte boundary:
// each lane moves 16 bytes per load, rows stay in registers between the amax and the
// quantisation, and nothing divides.  Bit-identical to the general kernels above (same
// exponent rule, same rounding).

template <typename InT> struct Vec16 {
  static constexpr int kN = 16 / sizeof(InT);          // elements per 16-byte vector
};

template <typename InT>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  const InT* e = reinterpret_cast<const InT*>(&u);
#pragma unroll
  for (int i = 0; i < Vec16<InT>::kN; ++i) f[i] = to_f32(e[i]);
}

// pack kN quantised values (bytes) into kN bytes: 8 -> uint2, 4 -> uint32
template <int N> struct PackOut;
template <> struct PackOut<8> {
  using T = uint2;
  static __device__ __forceinline__ T pack(const int* q) {
    T r;
    r.x = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) | ((uint32_t)q[3] << 24);
    r.y = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) | ((uint32_t)q[7] << 24);
    return r;
  }
};
template <> struct PackOut<4> {
  using T = uint32_t;
  static __device__ __forceinline__ T pack(const int* q) {
    return (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) | ((uint32_t)q[3] << 24);
  }
};

// P1 fast path: G = DH*sizeof/16 lanes per row, 32/G rows per warp, kRowsPerLane row groups per
// CTA pass (all their 16-byte loads are issued before any is used); `cta` = the 256-thread CTA's
// index in the row space.
constexpr int kRowsPerLane = 4;
template <typename InT, int DH>
__device__ __forceinline__ void quant_rows_vec(int cta, const InT* __restrict__ x, Strides4 xs, int B, int H, int T,
                                               int Tpad, int8_t* __restrict__ q8, int32_t* __restrict__ eq) {
  constexpr int N = Vec16<InT>::kN;
  constexpr int G = DH / N;                            // lanes per row
  constexpr int RPW = 32 / G;                          // rows per warp
  constexpr int RPC = 8 * RPW;                         // rows per CTA and row group
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const long long nrows = (long long)B * H * Tpad;
  const long long row0 = (long long)cta * RPC * kRowsPerLane + (threadIdx.x >> 5) * RPW + lane / G;
  uint4 u[kRowsPerLane];
  bool data[kRowsPerLane];
  if (Tpad % (RPC * kRowsPerLane) == 0) {
    // the CTA's rows lie in one window of one (b, h): one index computation per thread
    const long long rr0 = row0 < nrows ? row0 : 0;
    const int t0 = (int)(rr0 % Tpad);
    const long long bh = rr0 / Tpad;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const InT* xrow = x + b * xs.s0 + h * xs.s1 + sub * N;
#pragma unroll
    for (int k = 0; k < kRowsPerLane; ++k) {
      const long long row = row0 + (long long)k * RPC;
      const int t = t0 + k * RPC;
      data[k] = row < nrows && t < T;
      u[k] = data[k] ? *reinterpret_cast<const uint4*>(xrow + (long long)t * xs.s2) : make_uint4(0u, 0u, 0u, 0u);
    }
  } else {                                             // e.g. one row per (b, h) (decode queries)
#pragma unroll
    for (int k = 0; k < kRowsPerLane; ++k) {
      const long long row = row0 + (long long)k * RPC;
      const long long rr = row < nrows ? row : 0;
      const int t = (int)(rr % Tpad);
      const long long bh = rr / Tpad;
      const int h = (int)(bh % H), b = (int)(bh / H);
      data[k] = row < nrows && t < T;
      u[k] = data[k] ? *reinterpret_cast<const uint4*>(x + b * xs.s0 + h * xs.s1 + (long long)t * xs.s2 + sub * N)
                     : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int k = 0; k < kRowsPerLane; ++k) {
    const long long row = row0 + (long long)k * RPC;
    float f[N];
    unpack16<InT>(u[k], f);
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) m = fmaxf(m, fabsf(f[i]));
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (row < nrows) {
      const int e = data[k] ? pow2_exponent(m, 40) : 0;
      const float sc = pow2f(e);
      int q[N];
#pragma unroll
      for (int i = 0; i < N; ++i) q[i] = quant8(f[i], sc);     // rows past T: zeros
      *reinterpret_cast<typename PackOut<N>::T*>(q8 + row * DH + sub * N) = PackOut<N>::pack(q);
      if (sub == 0) eq[row] = e;
    }
  }
}

template <typename InT, int DH>
__global__ void __launch_bounds__(256)
quant_rows_vec_kernel(const InT* __restrict__ x, Strides4 xs, int B, int H, int T, int Tpad,
                      int8_t* __restrict__ q8, int32_t* __restrict__ eq) {
  pdl_launch_dependents();                             // a PDL-launched consumer may start its setup
  quant_rows_vec<InT, DH>((int)blockIdx.x, x, xs, B, H, T, Tpad, q8, eq);
  // launched with programmatic dependent launch after a kernel it does not read (the decode
  // plan), it still completes only after that kernel, so a consumer's wait on this grid covers
  // both (a no-op otherwise)
  pdl_wait();
}

// P2/P3 fast path: one CTA of 256 threads per (block, kv head, batch); the block's 128 x DH
// values stay in registers (<= 8 vectors per thread) between the amax and the quantisation.
template <typename InT, int DH>
__device__ __forceinline__ void quant_blocks_vec(int blk, int g, int b, const InT* __restrict__ x, Strides4 xs,
                                                 int B, int KVH, int T, int Tpad, int mode, int8_t* __restrict__ x8,
                                                 int32_t* __restrict__ eblk, int32_t* __restrict__ e0,
                                                 int* __restrict__ err) {
  constexpr int N = Vec16<InT>::kN;
  constexpr int VPR = DH / N;                          // vectors per row
  constexpr int VPT = 128 * VPR / 256;                 // vectors per thread
  const int nblk = (T + kKB - 1) / kKB;
  const int lo = blk * kKB;
  const int hi = min(T, lo + kKB);
  const bool split0 = (mode == 2) && (blk == 0) && (T > 1);
  const InT* src = x + b * xs.s0 + g * xs.s1;
  int8_t* dst = x8 + ((long long)(b * KVH + g) * Tpad) * DH;
  __shared__ float red[2][8];
  uint4 raw[VPT];                                      // raw 16-byte vectors: half the registers of floats
  float m = 0.0f, m0 = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * 256;
    const int r = lo + v / VPR, c = (v % VPR) * N;
    raw[i] = (r < hi) ? *reinterpret_cast<const uint4*>(src + (long long)r * xs.s2 + c) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * 256;
    const int r = lo + v / VPR;
    float f[N];
    unpack16<InT>(raw[i], f);
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < N; ++k) a = fmaxf(a, fabsf(f[k]));
    if (split0 && r == 0) m0 = fmaxf(m0, a); else m = fmaxf(m, a);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
  }
  if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = m; red[1][threadIdx.x >> 5] = m0; }
  __syncthreads();
  m = 0.0f; m0 = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) { m = fmaxf(m, red[0][w]); m0 = fmaxf(m0, red[1][w]); }
  const int hic = (mode == 0) ? 40 : 48;
  const int e = pow2_exponent(m, hic);
  const int ez = split0 ? pow2_exponent(m0, 48) : e;
  const float sc = pow2f(e), sc0 = pow2f(ez);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * 256;
    const int r = lo + v / VPR, c = (v % VPR) * N;
    if (r < lo + kKB && r < Tpad) {                    // rows past T (padding) become zeros
      float f[N];
      unpack16<InT>(raw[i], f);
      int q[N];
#pragma unroll
      for (int k = 0; k < N; ++k) q[k] = (r < hi) ? quant8(f[k], (split0 && r == 0) ? sc0 : sc) : 0;
      *reinterpret_cast<typename PackOut<N>::T*>(dst + (long long)r * DH + c) = PackOut<N>::pack(q);
    }
  }
  // zero padding rows past this (last) block, up to Tpad
  if (blk == nblk - 1) {
    const int npad = (Tpad - (lo + kKB)) * DH;
    for (int i = threadIdx.x; i < npad; i += blockDim.x) dst[(long long)(lo + kKB) * DH + i] = 0;
  }
  if (threadIdx.x == 0) {
    eblk[(long long)(b * KVH + g) * nblk + blk] = e;
    if (mode == 2 && blk == 0) e0[b * KVH + g] = ez;
    if (mode != 0 && (e < -32 || e > 40)) atomicOr(err, kDevEvRange);
  }
}

template <typename InT, int DH>
__global__ void __launch_bounds__(256)
quant_blocks_vec_kernel(const InT* __restrict__ x, Strides4 xs, int B, int KVH, int T, int Tpad, int mode,
                        int8_t* __restrict__ x8, int32_t* __restrict__ eblk, int32_t* __restrict__ e0,
                        int* __restrict__ err) {
  quant_blocks_vec<InT, DH>((int)blockIdx.x, (int)blockIdx.y, (int)blockIdx.z, x, xs, B, KVH, T, Tpad, mode, x8,
                            eblk, e0, err);
}

// The prefill's K and V quantisers in one launch (P2 for K, P2 or P3 for V): CTAs [0, nk)
// quantise K's (block, kv head, batch) tiles, CTAs [nk, 2 nk) V's.  (Q's row quantiser stays a
// separate kernel: fused, it would run at this kernel's register count and lose occupancy.)
template <typename InT, int DH>
__global__ void __launch_bounds__(256)
quant_kv_vec_kernel(const InT* __restrict__ k, Strides4 ks, const InT* __restrict__ v, Strides4 vs, int B, int KVH,
                    int T, int Tpad, int vmode, int8_t* __restrict__ k8, int32_t* __restrict__ ek,
                    int8_t* __restrict__ v8, int32_t* __restrict__ ev, int32_t* __restrict__ ev0,
                    int* __restrict__ err) {
  const int nblk = Tpad / kKB;
  const int nk = nblk * KVH * B;
  const int i = (int)blockIdx.x;
  const bool isv = i >= nk;
  const int j = isv ? i - nk : i;
  const int blk = j % nblk, g = (j / nblk) % KVH, b = j / (nblk * KVH);
  if (!isv) quant_blocks_vec<InT, DH>(blk, g, b, k, ks, B, KVH, T, Tpad, 0, k8, ek, ev0, err);
  else quant_blocks_vec<InT, DH>(blk, g, b, v, vs, B, KVH, T, Tpad, vmode, v8, ev, ev0, err);
  pdl_launch_dependents();                             // released as the CTAs finish
}

}  // namespace lssab8
