// LSSA-B8 split-KV decode on sm_100a (HBM-bound byte/integer work).
//
// The KV cache is a PAGED int8 lattice (16-key pages; a contiguous cache is the identity page
// table):
//   k8p [P, KVH, 16, dh]  key rows of a page, one kv head contiguous (2 KB at dh 128)
//   v8p [P, KVH, dh, 16]  the page's values TRANSPOSED (channel-major), so 4 consecutive keys
//                         of one channel are one 32-bit word for dp4a
//   ek, ev [B, KVH, max_blocks] int32 per logical 128-key block; ev0 [B, KVH] (B9.1 sink)
//
// One CTA = (split, kv head, sequence): the split's 128-key blocks stream through a 2-stage
// shared-memory ring with cp.async.bulk (16 page copies of 2 KB per block), the GQA group's
// query rows sit in shared memory, and for each block the CTA computes the EXACT integer block
// partials of every head of the group (docs/contract/BLOCK_EXPONENT_VARIANT.md B8.4):
//   S (int32, dp4a), block max, NB_b, the 32-bit chain and T2 gather, l_b, A_b = eh . v8
// and writes (A_b, NB_b, l_b, eh0) to the workspace.  A split below segment granularity may only
// exchange exact block partials (reference/lssab8_golden.py:350-394); the LAST CTA of a
// (sequence, kv head) to finish (an atomic ticket, no waiting) refolds all blocks in ascending
// order with the two-level committed-order fold and writes the output rows.
#pragma once
#include "tcgen05.cuh"

namespace lssab8 {

struct DecodeArgs {
  int B, H, KVH, dh, group;          // group = H / KVH (<= 8)
  int max_blocks;                     // exponent / partial array extent per (b, g)
  int max_pages;                      // block_table row length
  int split_blocks;                   // blocks per split
  int num_pages;                      // physical pool size (for bounds checks)
  const int32_t* seq_lens;            // [B]
  const int32_t* block_table;         // [B, max_pages]
  const int8_t* k8p;                  // [P, KVH, 16, dh]
  const int8_t* v8p;                  // [P, KVH, dh, 16]
  const int32_t* ek;                  // [B, KVH, max_blocks]
  const int32_t* ev;
  const int32_t* ev0;                 // [B, KVH] or nullptr (sink off)
  const int8_t* q8;                   // [B, H, dh]
  const int32_t* eq;                  // [B, H]
  int32_t* partA;                     // [B, KVH, max_blocks, group, dh]
  int4* partM;                        // [B, KVH, max_blocks, group] {nb, l_b, eh0, 0}
  unsigned int* tickets;              // [B, KVH], zero before the launch (dh 64)
  int* blk_off;                       // [B + 1] live blocks of the sequences before b (dh 128)
  int* order;                         // [B] the refold's sequence order, longest first (dh 128)
  void* out; long long os0, os1, os2; // out[b, h, c]
  uint32_t gbase;
  int* err;
};

__device__ __forceinline__ uint32_t dp4a_us(uint32_t a_u8x4, uint32_t b_s8x4, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8x4), "r"(b_s8x4), "r"(c));
  return d;
}

template <int DH>
struct DecodeSmem {
  static constexpr int kPage = 16 * DH;                 // bytes of one page, one kv head
  static constexpr int kStage = 2 * 8 * kPage;          // K block + V block
  static constexpr int kK = 0;                          // stage s: K at s*kStage, V at s*kStage + 8*kPage
  static constexpr int kTab = 2 * kStage;
  static constexpr int kQ = kTab + kTabPad;             // [8][DH] int8
  static constexpr int kEh = kQ + 8 * DH;               // [8][128] u8
  static constexpr int kRed = kEh + 8 * 128;            // 80 ints: max[4][8], l_b[4][8], eh0[8], nb[8]
  static constexpr int kBar = kRed + 384;
  static constexpr int kBytes = kBar + 64;
};

// The committed-order refold of head h of one (sequence, kv head) from its exact block partials,
// for channel c: blocks in ascending order into 32-block segments, segments into the row
// (reference/lssab8_golden.py:350-394, 257-335), then one RN division.  kBatch blocks' partial
// loads are issued before any is used, so their latencies overlap; partials are read with .cg
// loads (other CTAs wrote them).
template <int DH, bool SINK, typename OutT, int kBatch>
__device__ __forceinline__ void decode_merge_head(const DecodeArgs& p, int b, int g, int h, int c) {
  const int gq = p.group;
  const int L_len = p.seq_lens[b];
  const int nblk = (L_len + kKB - 1) / kKB;
  const long long bg = (long long)b * p.KVH + g;
  int v0c = 0, evs0 = 0, eh0 = 0;
  if (SINK && L_len > 1) {
    const int pg = p.block_table[(long long)b * p.max_pages];
    v0c = (int)p.v8p[((long long)pg * p.KVH + g) * (16 * DH) + c * 16 + 0];
    evs0 = p.ev0[bg];
    eh0 = __ldcg(&p.partM[(bg * p.max_blocks) * gq + h]).z;
  }
  float Orow = 0.0f, lrow = 0.0f;
  int nbrow = 0;
  for (int s0 = 0; s0 < nblk; s0 += kSEG) {
    const int s1 = min(nblk, s0 + kSEG);
    float O = 0.0f, lseg = 0.0f;
    int nbrun = 0;
    for (int k0 = s0; k0 < s1; k0 += kBatch) {
      int2 m2[kBatch];                                   // (NB_b, l_b)
      int Av[kBatch], evv[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int blk = min(k0 + u, s1 - 1);
        evv[u] = p.ev[bg * p.max_blocks + blk];
        m2[u] = __ldcg(reinterpret_cast<const int2*>(&p.partM[(bg * p.max_blocks + blk) * gq + h]));
        Av[u] = __ldcg(&p.partA[((bg * p.max_blocks + blk) * gq + h) * DH + c]);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int blk = k0 + u;
        if (blk >= s1) break;
        if (blk == s0) nbrun = m2[u].x;
        const int D = m2[u].x - nbrun;
        int sg = 0;
        if (D > 0) { O = rescale(O, D); lseg = rescale(lseg, D); nbrun = m2[u].x; }
        else sg = -D;
        if (sg <= kSWIN) {
          if (SINK && blk == 0 && L_len > 1) O = fold_term(O, eh0 * v0c, pow2f(-(sg + evs0)));
          O = fold_term(O, Av[u], pow2f(-(sg + evv[u])));
          lseg = fold_term(lseg, m2[u].y, pow2f(-sg));
        }
      }
    }
    // segment -> row (reference/lssab8_golden.py:317-331)
    if (s0 == 0) nbrow = nbrun;
    const int D2 = nbrun - nbrow;
    int s2 = 0;
    if (D2 > 0) { Orow = rescale(Orow, D2); lrow = rescale(lrow, D2); nbrow = nbrun; }
    else s2 = -D2;
    if (s2 <= kSWIN) {
      Orow = __fadd_rn(Orow, rescale(O, s2));
      lrow = __fadd_rn(lrow, rescale(lseg, s2));
    }
  }
  const float y = (lrow != 0.0f) ? __fdiv_rn(Orow, lrow) : 0.0f;
  OutT* dst = reinterpret_cast<OutT*>(p.out) + b * p.os0 + (long long)(g * gq + h) * p.os1 + c * p.os2;
  *dst = from_f32<OutT>(y);
}

template <int DH, bool SINK, typename OutT>
__global__ void __launch_bounds__(128)
decode_kernel(const DecodeArgs p) {
  using L = DecodeSmem<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);        // 128-B aligned, still __shared__
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint8_t* tab = smem + L::kTab;
  int8_t* sq = reinterpret_cast<int8_t*>(smem + L::kQ);
  uint8_t* seh = smem + L::kEh;
  int* red = reinterpret_cast<int*>(smem + L::kRed);
  __shared__ int s_last;
  __shared__ int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int gq = p.group;
  const int L_len = p.seq_lens[b];
  const int nblk = (L_len + kKB - 1) / kKB;
  const int nsplit = (nblk + p.split_blocks - 1) / p.split_blocks;
  if (L_len <= 0 || split >= nsplit) return;
  if (nblk > p.max_blocks || (L_len + 15) / 16 > p.max_pages) {   // lattice arrays too short
    if (tid == 0) atomicOr(p.err, kDevBadPage);
    return;
  }
  const int blo = split * p.split_blocks;
  const int bhi = min(nblk, blo + p.split_blocks);
  const long long bg = (long long)b * p.KVH + g;
  const int32_t* bt = p.block_table + (long long)b * p.max_pages;

  for (int i = tid; i < kTabPad; i += blockDim.x) tab[i] = (i < kTabLive) ? kT2Live[i] : 0;
  for (int i = tid; i < gq * DH; i += blockDim.x) sq[i] = p.q8[((long long)b * p.H + g * gq) * DH + i];
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // issue the page copies of logical block blk into stage s (thread 0 only)
  auto issue = [&](int blk, int s) {
    uint8_t* kdst = smem + s * L::kStage;
    uint8_t* vdst = kdst + 8 * L::kPage;
    const int pg0 = blk * 8;
    const int npg = min(8, (L_len - blk * kKB + 15) / 16);
    mbar_expect_tx(&bars[s], (uint32_t)(2 * npg * L::kPage));
    for (int i = 0; i < npg; ++i) {
      int pg = bt[pg0 + i];
      if (pg < 0 || pg >= p.num_pages) { atomicOr(p.err, kDevBadPage); pg = 0; }
      const long long off = ((long long)pg * p.KVH + g) * L::kPage;
      bulk_g2s(kdst + i * L::kPage, p.k8p + off, L::kPage, &bars[s]);
      bulk_g2s(vdst + i * L::kPage, p.v8p + off, L::kPage, &bars[s]);
    }
  };
  if (tid == 0) {
    issue(blo, 0);
    if (blo + 1 < bhi) issue(blo + 1, 1);
  }

  for (int blk = blo; blk < bhi; ++blk) {
    const int j = blk - blo;
    const int s = j & 1;
    const uint32_t ph = (j >> 1) & 1;
    if (!mbar_wait(&bars[s], ph, &s_abort, p.err)) break;
    const uint8_t* kblk = smem + s * L::kStage;
    const uint8_t* vblk = kblk + 8 * L::kPage;
    const int nkeys = min(kKB, L_len - blk * kKB);
    // ---- scores: thread t = key t, every head of the group
    int S[8];
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) S[hh] = 0;
    if (tid < nkeys) {
      const uint8_t* krow = kblk + tid * DH;
#pragma unroll
      for (int k = 0; k < DH / 16; ++k) {
        const int ch = (k + tid) & (DH / 16 - 1);            // rotate chunks: conflict-free
        const uint4 kw = *reinterpret_cast<const uint4*>(krow + ch * 16);
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) {
          if (hh < gq) {
            const uint4 qw = *reinterpret_cast<const uint4*>(sq + hh * DH + ch * 16);
            S[hh] = __dp4a((int)kw.x, (int)qw.x, S[hh]);
            S[hh] = __dp4a((int)kw.y, (int)qw.y, S[hh]);
            S[hh] = __dp4a((int)kw.z, (int)qw.z, S[hh]);
            S[hh] = __dp4a((int)kw.w, (int)qw.w, S[hh]);
          }
        }
      }
    } else {
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) S[hh] = INT32_MIN;     // keys past the sequence end
    }
    // ---- block max per head (exact, order-free)
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) {
      if (hh < gq) {
        int m = S[hh];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp * 8 + hh] = m;
      }
    }
    __syncthreads();
    // ---- chain: eh for (head, key t), l_b per head
    const int ekb = p.ek[bg * p.max_blocks + blk];
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) {
      if (hh < gq) {
        const int m = max(max(red[hh], red[8 + hh]), max(red[16 + hh], red[24 + hh]));
        const uint32_t G = g_fold(p.gbase, p.eq[(long long)b * p.H + g * gq + hh] + ekb);
        const int nbv = nb_of(m, G);
        const uint32_t NBlo = (uint32_t)nbv << kBHI;
        const int dm = 1 << max(0, 30 - (31 - __clz((int)G)));
        const int sc = max(S[hh], m - dm);
        const uint32_t d = NBlo + (uint32_t)sc * (0u - G);
        uint32_t e = tab[d >> kIdxShift];
        int lbw = (int)e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lbw += __shfl_xor_sync(0xffffffffu, lbw, o);
        if (lane == 0) red[32 + warp * 8 + hh] = lbw;      // second reduction area
        if (SINK && blk == 0 && tid == 0 && L_len > 1) {
          red[64 + hh] = (int)e;                          // eh0, kept out of the PV product
          e = 0;
        }
        seh[hh * 128 + tid] = (uint8_t)e;
        if (tid == 0) red[72 + hh] = nbv;
      }
    }
    __syncthreads();
    // ---- PV: thread c = channel, A[hh] = sum_k eh[hh][k] * v8[k][c] (exact int32)
    if (tid < DH) {
      int A[8];
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) A[hh] = 0;
      const int npg = (nkeys + 15) / 16;
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int pgi = (i + tid) & 7;                       // rotate pages: conflict-free
        if (pgi >= npg) continue;
        const uint4 vw = *reinterpret_cast<const uint4*>(vblk + pgi * L::kPage + tid * 16);
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) {
          if (hh < gq) {
            const uint4 ew = *reinterpret_cast<const uint4*>(seh + hh * 128 + pgi * 16);
            uint32_t a = (uint32_t)A[hh];
            a = dp4a_us(ew.x, vw.x, a);
            a = dp4a_us(ew.y, vw.y, a);
            a = dp4a_us(ew.z, vw.z, a);
            a = dp4a_us(ew.w, vw.w, a);
            A[hh] = (int)a;
          }
        }
      }
      int32_t* dstA = p.partA + ((bg * p.max_blocks + blk) * gq) * DH;
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) if (hh < gq) dstA[hh * DH + tid] = A[hh];
    }
    if (tid < gq) {
      const int hh = tid;
      const int lb = red[32 + hh] + red[40 + hh] + red[48 + hh] + red[56 + hh];
      const int e0 = (SINK && blk == 0 && L_len > 1) ? red[64 + hh] : 0;
      p.partM[(bg * p.max_blocks + blk) * gq + hh] = make_int4(red[72 + hh], lb, e0, 0);
    }
    __syncthreads();                                         // stage s and red/seh are free
    if (tid == 0 && blk + 2 < bhi) issue(blk + 2, s);
  }

  // ---- ticket: the last split of this (sequence, kv head) merges, in ascending block order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int t = atomicAdd(&p.tickets[bg], 1u);
    s_last = (t == (unsigned int)(nsplit - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) p.tickets[bg] = 0u;                          // ready for the next launch
  if (tid >= DH) return;
  for (int hh = 0; hh < gq; ++hh) decode_merge_head<DH, SINK, OutT, 8>(p, b, g, hh, tid);
}

// Decode lattice writer: quantise a sequence's K and V (bf16/f16/f32, any strides) into the
// paged lattice.  One CTA per (logical block, kv head, sequence); the block exponent is over
// the block's present rows (reference/lssab_torch.py:62-85); with the sink on, key 0 is
// quantised alone and block 0's value exponent covers keys 1.. (reference/lssab9_torch.py:124-132).
// Source element (b, t, g, c) is at src + seq_off[b] + t*st + g*sg + c*sc.
template <typename InT>
__global__ void __launch_bounds__(256)
decode_prep_kernel(const InT* __restrict__ ksrc, const InT* __restrict__ vsrc, const long long* __restrict__ seq_off,
                   long long st, long long sg, long long sc, int B, int KVH, int dh, const int32_t* __restrict__ seq_lens,
                   const int32_t* __restrict__ block_table, int max_pages, int max_blocks, int num_pages, int vmode,
                   int8_t* __restrict__ k8p, int8_t* __restrict__ v8p, int32_t* __restrict__ ek, int32_t* __restrict__ ev,
                   int32_t* __restrict__ ev0, int* __restrict__ err) {
  const int blk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int L_len = seq_lens[b];
  const int nblk = (L_len + kKB - 1) / kKB;
  if (blk >= nblk) return;
  if (nblk > max_blocks || (L_len + 15) / 16 > max_pages) {        // lattice arrays too short
    if (threadIdx.x == 0) atomicOr(err, kDevBadPage);
    return;
  }
  const int lo = blk * kKB, hi = min(L_len, lo + kKB);
  const int n = (hi - lo) * dh;
  __shared__ float red[4][8];
  const long long base = seq_off[b] + g * sg;
  const int32_t* bt = block_table + (long long)b * max_pages;
  for (int which = 0; which < 2; ++which) {
    const InT* src = (which == 0) ? ksrc : vsrc;
    const int mode = (which == 0) ? 0 : vmode;
    const bool split0 = (mode == 2) && (blk == 0) && (L_len > 1);
    float m = 0.0f, m0 = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int r = lo + i / dh, c = i % dh;
      const float a = fabsf(to_f32(src[base + (long long)r * st + (long long)c * sc]));
      if (split0 && r == 0) m0 = fmaxf(m0, a); else m = fmaxf(m, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    }
    if ((threadIdx.x & 31) == 0) { red[which * 2][threadIdx.x >> 5] = m; red[which * 2 + 1][threadIdx.x >> 5] = m0; }
    __syncthreads();
    m = 0.0f; m0 = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { m = fmaxf(m, red[which * 2][w]); m0 = fmaxf(m0, red[which * 2 + 1][w]); }
    const int e = pow2_exponent(m, mode == 0 ? 40 : 48);
    const int ez = split0 ? pow2_exponent(m0, 48) : e;
    const float scl = pow2f(e), scl0 = pow2f(ez);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int r = lo + i / dh, c = i % dh;
      const float x = to_f32(src[base + (long long)r * st + (long long)c * sc]);
      const int q = quant8(x, (split0 && r == 0) ? scl0 : scl);
      int pg = bt[r >> 4];
      if (pg < 0 || pg >= num_pages) { atomicOr(err, kDevBadPage); continue; }
      const long long pbase = ((long long)pg * KVH + g) * 16 * dh;
      if (which == 0) k8p[pbase + (r & 15) * dh + c] = (int8_t)q;
      else v8p[pbase + c * 16 + (r & 15)] = (int8_t)q;
    }
    // zero the unused rows of the last page so the bulk copies read defined bytes
    if (blk == nblk - 1 && (hi & 15)) {
      int pg = bt[(hi - 1) >> 4];
      if (pg >= 0 && pg < num_pages) {
        const long long pbase = ((long long)pg * KVH + g) * 16 * dh;
        const int nz = (16 - (hi & 15)) * dh;
        for (int i = threadIdx.x; i < nz; i += blockDim.x) {
          const int rr = (hi & 15) + i / dh, c = i % dh;
          if (which == 0) k8p[pbase + rr * dh + c] = 0;
          else v8p[pbase + c * 16 + rr] = 0;
        }
      }
    }
    if (threadIdx.x == 0) {
      const long long o = ((long long)b * KVH + g) * max_blocks + blk;
      if (which == 0) ek[o] = e;
      else {
        ev[o] = e;
        if (mode == 2 && blk == 0) ev0[(long long)b * KVH + g] = ez;
        if (mode != 0 && (e < -32 || e > 40)) atomicOr(err, kDevEvRange);
      }
    }
    __syncthreads();
  }
}

// The paged lattice writer, vectorised, with append-only semantics (the engine's per-step prep,
// docs/contract/BLOCK_EXPONENT_VARIANT.md:53-55, 212-215: a complete 128-key block never changes;
// the open block's exponents and values are recomputed from its present rows).  One CTA per
// (128-key block, kv head, sequence, tensor): K and V blocks are separate CTAs (their exponents are
// independent).  Blocks below start_lens[b] / 128 (complete before this append) are left as they
// are.  Thread (pl, cv) holds page pl of the block (16 keys) x channels [cv EPV, cv EPV + EPV) in
// registers, read once as 16 16-byte vectors, for the amax and the quantisation; only the block
// maximum passes through shared memory.  A K page row is 8 (bf16) bytes per thread, stored as it
// is; a V page is the transposed [channel][16 keys], so each of the thread's channels becomes one
// 16-byte row packed in registers.  Token t of sequence b, kv head g, channel c is read at
//   src + seq_off[b] + t * st + g * sg + c                 (src_bt == nullptr), or
//   src + src_bt[b, t / 16] * src_ps + (t % 16) * st + g * sg + c  (a paged source cache whose
//                                                           page ids are below num_pages).
// Rows past the sequence end inside its last page are written as zeros.
template <typename InT, int DH>
struct KvLattice {
  static constexpr int kEpv = 16 / (int)sizeof(InT);        // channels per 16-byte vector
  static constexpr int kVpr = DH / kEpv;                    // vectors per key row
  static constexpr int kThreads = 8 * kVpr;                 // 8 pages x kVpr
};

// four int8 values (clamped to [-127, 127]) packed into one word, lowest first
__device__ __forceinline__ uint32_t pack4_s8(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// max |x| over a 16-byte vector, on the bit patterns: with the sign cleared a pattern is monotone
// in |x| (zeros, subnormals and infinity included), and a NaN (a pattern above infinity's) counts
// as 0, which is fmaxf's rule of ignoring NaN.  acc holds the running maximum pattern(s): two
// 16-bit lanes for bf16 / fp16, one word for f32; absmax_value turns it into the float.
template <typename InT>
__device__ __forceinline__ uint32_t absmax_acc(uint32_t acc, const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (sizeof(InT) == 2) {
    constexpr uint32_t kInf2 = std::is_same<InT, __half>::value ? 0x7C007C00u : 0x7F807F80u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = w[i] & 0x7FFF7FFFu;
      acc = __vmaxu2(acc, a & ~__vcmpgtu2(a, kInf2));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = w[i] & 0x7FFFFFFFu;
      acc = max(acc, a > 0x7F800000u ? 0u : a);
    }
  }
  return acc;
}
template <typename InT>
__device__ __forceinline__ float absmax_value(uint32_t acc) {
  if constexpr (sizeof(InT) == 2) {
    const uint32_t h = max(acc & 0xFFFFu, acc >> 16);
    if constexpr (std::is_same<InT, __half>::value) return __half2float(__ushort_as_half((unsigned short)h));
    else return __uint_as_float(h << 16);
  } else {
    return __uint_as_float(acc);
  }
}

template <typename InT, int DH>
__global__ void __launch_bounds__(KvLattice<InT, DH>::kThreads)
kv_lattice_kernel(const InT* __restrict__ ksrc, const InT* __restrict__ vsrc, const long long* __restrict__ seq_off,
                  long long st, long long sg, const int32_t* __restrict__ src_bt, long long src_ps, int B, int KVH,
                  const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ start_lens,
                  const int32_t* __restrict__ block_table, int max_pages, int max_blocks, int num_pages, int vmode,
                  int8_t* __restrict__ k8p, int8_t* __restrict__ v8p, int32_t* __restrict__ ek,
                  int32_t* __restrict__ ev, int32_t* __restrict__ ev0, int* __restrict__ err) {
  using K = KvLattice<InT, DH>;
  constexpr int EPV = K::kEpv, VPR = K::kVpr, NW = K::kThreads / 32;
  const int blk = blockIdx.x, g = blockIdx.y, b = blockIdx.z >> 1;
  const bool isv = (blockIdx.z & 1) != 0;                // this CTA's tensor: K (0) or V (1)
  const int L = seq_lens[b];
  const int nblk = (L + kKB - 1) / kKB;
  if (blk >= nblk) return;
  if (nblk > max_blocks || (L + 15) / 16 > max_pages) {
    if (threadIdx.x == 0 && !isv) atomicOr(err, kDevBadPage);
    return;
  }
  if (start_lens && blk < start_lens[b] / kKB) return;   // complete before this append: unchanged
  const int pl = threadIdx.x / VPR, cv = threadIdx.x % VPR;
  const int lo = blk * kKB + pl * 16;                    // this thread's first key
  const int npages = min(8, ((L + 15) / 16) - blk * 8);  // pages of this block that exist
  const int32_t* bt = block_table + (long long)b * max_pages;
  const InT* src = isv ? vsrc : ksrc;
  __shared__ float red[2][NW];
  const bool split0 = isv && (vmode == 2) && (blk == 0) && (L > 1);   // key 0 alone (B9.1)
  bool have = lo < L;
  long long rb = 0;                                      // element offset of key lo, channel cv EPV
  if (have) {
    if (src_bt) {
      const int sp = src_bt[(long long)b * max_pages + blk * 8 + pl];
      if (sp < 0 || sp >= num_pages) { atomicOr(err, kDevBadPage); have = false; }
      else rb = (long long)sp * src_ps + g * sg + cv * EPV;
    } else {
      rb = seq_off[b] + (long long)lo * st + g * sg + cv * EPV;
    }
    if (rb & (EPV - 1)) { atomicOr(err, kDevAlign); have = false; }   // a row off the 16-byte grid
  }
  uint4 x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    x[i] = make_uint4(0u, 0u, 0u, 0u);
    if (have && lo + i < L) x[i] = __ldg(reinterpret_cast<const uint4*>(src + rb + i * st));
  }
  uint32_t am = 0u, am0 = 0u;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i == 0 && split0 && pl == 0) am0 = absmax_acc<InT>(0u, x[0]);
    else am = absmax_acc<InT>(am, x[i]);
  }
  float m = absmax_value<InT>(am), m0 = absmax_value<InT>(am0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { red[0][w] = m; red[1][w] = m0; }
  __syncthreads();
  m = red[0][0]; m0 = red[1][0];
#pragma unroll
  for (int i = 1; i < NW; ++i) { m = fmaxf(m, red[0][i]); m0 = fmaxf(m0, red[1][i]); }
  const int e1 = pow2_exponent(m, (!isv || vmode == 0) ? 40 : 48);
  const int e0 = split0 ? pow2_exponent(m0, 48) : e1;
  const float s1 = pow2f(e1), s0 = pow2f(e0);
  if (pl < npages) {                                     // the page exists
    const int pg = bt[blk * 8 + pl];
    if (pg < 0 || pg >= num_pages) {
      atomicOr(err, kDevBadPage);
    } else if (!isv) {                                   // K page [16 keys][DH]: this thread's EPV channels of each key
      int8_t* kd = k8p + ((long long)pg * KVH + g) * 16 * DH + cv * EPV;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const InT* xe = reinterpret_cast<const InT*>(&x[i]);
        uint32_t kq[EPV / 4];
#pragma unroll
        for (int q = 0; q < EPV / 4; ++q)
          kq[q] = pack4_s8(quant8(to_f32(xe[4 * q]), s1), quant8(to_f32(xe[4 * q + 1]), s1),
                           quant8(to_f32(xe[4 * q + 2]), s1), quant8(to_f32(xe[4 * q + 3]), s1));
        if constexpr (EPV == 8) *reinterpret_cast<uint2*>(kd + i * DH) = make_uint2(kq[0], kq[1]);
        else *reinterpret_cast<uint32_t*>(kd + i * DH) = kq[0];
      }
    } else {                                             // V page [DH][16 keys]: one 16-byte row per channel
      int8_t* vd = v8p + (((long long)pg * KVH + g) * DH + cv * EPV) * 16;
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        int q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          q[i] = quant8(to_f32(reinterpret_cast<const InT*>(&x[i])[e]), (i == 0 && split0 && pl == 0) ? s0 : s1);
        *reinterpret_cast<uint4*>(vd + e * 16) = make_uint4(pack4_s8(q[0], q[1], q[2], q[3]), pack4_s8(q[4], q[5], q[6], q[7]),
                                                           pack4_s8(q[8], q[9], q[10], q[11]),
                                                           pack4_s8(q[12], q[13], q[14], q[15]));
      }
    }
  }
  if (threadIdx.x == 0) {
    const long long o = ((long long)b * KVH + g) * max_blocks + blk;
    if (!isv) {
      ek[o] = e1;
    } else {
      ev[o] = e1;
      if (vmode == 2 && blk == 0) ev0[(long long)b * KVH + g] = e0;
      if (vmode != 0 && (e1 < -32 || e1 > 40)) atomicOr(err, kDevEvRange);
    }
  }
}

}  // namespace lssab8
