// LSSA-B8 causal / GQA prefill on sm_100a: tcgen05 int8 MMA with TMEM accumulators.
//
// Persistent: one CTA per SM walks the (query tile, batch, head) work items, longest tiles first
// in snake order, and for each item the key blocks 0 .. tile ASCENDING (the contract's
// committed order; a descending walk is a different function,
// docs/contract/BLOCK_EXPONENT_VARIANT.md B8.6).  Every pipeline (the TMA ring, S, P, A) runs on
// counters that continue across items, so the next item's loads and QK overlap this item's
// last folds and epilogue, and the setup (T2 copies, barriers, TMEM) is paid once per SM.
// A block-aligned chunk of query rows [128 tile0, T) runs the same way: query tile t of the chunk
// is key block tile0 + t of the sequence, and walks key blocks 0 .. tile0 + t.
// Warp-specialised roles:
//
//   warp 0      TMA producer: per item the Q tile (double-buffered across items) and key 0's
//               value row, then K/V 128-key blocks into a 2-stage ring (plain
//               cp.async.bulk.tensor, no multicast).
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_b  = Q8 . K8_b^T   tcgen05.mma kind::i8, s8 x s8 -> s32, M=128 N=128 K=dh
//                 A_b  = P_b . V8_b    tcgen05.mma kind::i8, u8 x s8 -> s32, M=128 N=dh K=128
//               TMEM columns: S [0, 128) (single: the chain copies a tile into registers
//               and releases it at once, so QK(j+1) overwrites it while block j's chain
//               runs), A double-buffered [128, 384) (PV(j+1) overlaps the fold of block j),
//               O [384, 512).  The kernel for rows that span more than one 32-block fold
//               segment (MULTI) keeps the row accumulator O_row in TMEM instead of A's second
//               buffer: A single [128, 256), O_row [256, 384), O_seg [384, 512); a single A
//               suffices because PV(j) is issued as soon as the fold of j - 1 (the same
//               iteration's second half) has released A, a whole chain before the fold of j.
//   warps 2-9   row workers, two threads per query row (TMEM lane = row).  Iteration j:
//               the chain of block j over this thread's 64 keys -- exact block max (the two
//               halves meet through shared memory at one named barrier per block), G, NB, the
//               32-bit chain d = NB - max(S, m - dm) * G (mod 2^32), the T2 gather from a
//               lane-replicated shared table (at most 2-way bank conflicts), l_b, and the u8 P
//               half-row in the SW128 K-major layout the PV MMA reads -- then the fold of block
//               j - 1 over this thread's DH/2 channels: the committed-order binary32 fold of
//               (NB_b, l_b, A_b) into the row's O, which lives in TMEM (paired f32x2
//               arithmetic), the segment -> row fold at 32-block boundaries (TMEM to TMEM), and
//               finally fl(O / l).
//               One role per SMSP-resident warp keeps the fold from being starved of issue
//               slots by separate chain warps, and 10 warps leave 168 registers per thread.
//
// The A accumulator is pre-loaded with the bit pattern 0x4B400000 (the float 1.5 * 2^23) and
// the PV MMA accumulates onto it, so the fold reads 1.5 * 2^23 + A_b as a float: one subtraction
// recovers A_b exactly (|A_b| < 2^22) and one fused multiply-add folds it (exact product, one
// rounding).  The MMA thread writes the bias before every PV with tcgen05.cp from a 4 KB block
// of bias words in shared memory, so the row workers spend no instructions on it.
//
// The general form (GEN, float32 output only) serves the golden entry points: p.causal = 0 lets
// every query tile walk every key block, and the key mask p.kmask (bit j of word j / 32 of the
// batch element's row: key j visible) hides keys from every row, as the golden's key_valid does
// (reference/lssab8_golden.py:241-247).  A row for which a whole block is hidden skips that block
// (no running-maximum update, no term), and a segment without a visible block skips the
// segment -> row step; a row that sees no key at all yields 0.
//
// B9.3 (KS kernels, v_keyshift; reference/lssab9_golden.py:179-186, reference/lssab9_torch.py:
// 145-153): key j's value row sits on the finer grid e_v + d_j (p.d8), so its PV weight is
// eh_j >> d_j while l_b keeps the unshifted eh_j; the chain packs both byte vectors.
//
// Exactness: S and A_b are exact integer sums (any MMA order); everything after them is the
// contract's integer chain and a fixed sequence of RN binary32 operations per row
// (reference/lssab8_torch.py:203-271, reference/lssab8_golden.py:257-335).  B9.1 sink_alone
// (reference/lssab9_torch.py:276-304): key 0's weight is removed from block 0's P operand
// (l_b keeps it) and its product eh0 * v8[0] is folded first with e_v0.
#pragma once
#include "tcgen05.cuh"

namespace lssab8 {
constexpr int kMaxPeers = 7;                                  // other ranks of one 8-GPU node
struct PrefillArgs {
  int B, H, KVH, T, dh, Tpad, nblk, group;
  int tile0;            // key-block index of the first query tile (a block-aligned chunk; 0: whole prefill)
  const int32_t* eq;    // [B, H, Tpad]
  const int32_t* ek;    // [B, KVH, nblk]
  const int32_t* ev;    // [B, KVH, nblk]
  const int32_t* ev0;   // [B, KVH] (sink) or nullptr
  const int8_t* v8;     // [B, KVH, Tpad, dh] (sink: key 0's row)
  void* out;            // output, element strides below
  long long os0, os1, os2, os3;   // out[b, t, h, c]
  int out_dtype;
  float* orow;          // unused (the row accumulator lives in TMEM); kept for the ABI
  uint32_t gbase;
  // Integer multipliers passed at run time (64, 2^8, 2^16, 2^24): the table address and the P
  // byte packing then compile to integer multiply-adds on the FMA pipe instead of shifts and
  // byte permutes on the ALU pipe, which the chain saturates.
  uint32_t mul_entry, mul_b1, mul_b2, mul_b3;
  int* err;
  uint64_t wait_ns;     // limit of every bounded wait (kWaitLimitNs; shorter only in the timeout self-test)
  int withhold;         // self-test only: the TMA producer never loads this key block of its first item (-1: none)
  // Peer outputs (the sharded prefill's gather): the same output rows are also stored, with the
  // same element strides, at each of these addresses -- other GPUs' output buffers mapped into
  // this process (CUDA IPC, P2P over NVLink) -- so every rank ends with every rank's heads.
  int npeers;
  void* peers[kMaxPeers];
  // the general form (GEN kernels): causal flag and key mask [B, nblk * 4] words
  int causal;
  const uint32_t* kmask;
  const int8_t* d8;     // B9.3 (KS kernels): per-key weight shift [B, KVH, nblk * 128]
};

// ------------------------------------------------------------------------ smem layout
constexpr int kTabCopies = 16;                                // T2 copies, one per lane of a half-warp
constexpr int kTabEntries = kTabLive + 1;                     // index 1152 (T2 = 0) absorbs clamped d
constexpr uint32_t kDClamp = (uint32_t)kTabLive << kIdxShift; // min(d, 1152 << 19) -> index <= 1152
constexpr uint32_t kMagicBits = 0x4B400000u;                  // 1.5 * 2^23
constexpr int kPrefillThreads = 320;                          // 10 warps: TMA, MMA, 8 row workers
constexpr int kTabBytes = kTabEntries * kTabCopies * 4;       // 73,792 B at the start of dynamic smem

template <int DH>
struct PrefillSmem {
  static constexpr int kTile = 128 * DH;                 // one Q/K/V tile, bytes
  static constexpr int kQ = 0;                           // 2 items
  static constexpr int kK = 2 * kTile;                   // 2 stages
  static constexpr int kV = 4 * kTile;                   // 2 stages
  static constexpr int kP = 6 * kTile;                   // 2 x 16 KB, SW128 K-major u8
  static constexpr int kV0 = kP + 2 * 16384;             // 2 items x key 0's int8 value row (sink)
  static constexpr int kMagic = kV0 + 2 * 128;           // 4 KB of the A bias words (tcgen05.cp source)
  static constexpr int kBar = kMagic + 4096;             // mbarriers
  static constexpr int kMisc = kBar + 256;               // tmem base, abort flag
  static constexpr int kBytes = kMisc + 64;              // (+ the static T2 table)
};

enum BarId : int {
  kBarQFull = 0, kBarKFull = 2, kBarKEmpty = 4, kBarVFull = 6, kBarVEmpty = 8, kBarSFull = 10, kBarSEmpty = 11,
  kBarPFull = 12, kBarPEmpty = 14, kBarAFull = 16, kBarAEmpty = 18, kBarQEmpty = 20
};

// Work item i (i = 0 .. ntile * B * H - 1), longest first: query tile ntile - 1 - i / (B * H),
// (b, h) = i % (B * H).  CTA k takes items r * G + k in even rounds r and r * G + G - 1 - k in odd
// rounds (snake order, G = gridDim.x), which balances the decreasing item sizes.
struct PfItem {
  int tile, b, h;
  int kt;               // the tile's key-block index: tile0 + tile (the diagonal block)
};
__device__ __forceinline__ bool pf_item(const PrefillArgs& p, int ntile, int round, PfItem& it) {
  const int G = gridDim.x;
  const int i = round * G + ((round & 1) ? (G - 1 - (int)blockIdx.x) : (int)blockIdx.x);
  if (i >= ntile * p.B * p.H) return false;
  const int bh = i % (p.B * p.H);
  it.tile = ntile - 1 - i / (p.B * p.H);
  it.kt = p.tile0 + it.tile;
  it.b = bh / p.H;
  it.h = bh % p.H;
  return true;
}
// TMEM column map: S, A (two buffers of 128; one in the MULTI kernel), O_row (MULTI), O (O_seg)
constexpr uint32_t kColS = 0, kColA = 128, kColOrow = 256, kColO = 384;

// The fold's running-maximum rescale of N channels (binary32 bit patterns) of one row by D > 0
// (reference/lssab8_golden.py:293-301; D <= 0 leaves them alone).  sD2 = (2^-min(D, 126)) twice.
// D <= 126: one paired multiply rounded toward zero with flush to zero per two channels -- the
// contract's exponent-field rescale except that a flushed negative value becomes -0, not +0; the
// caller adds a term with a positive scale next, which makes it +0.  D > 126: the
// compare-and-select form.  Register arithmetic only, so it may sit under per-row branches.
template <int N>
__device__ __forceinline__ void rescale_channels(uint32_t* o, int D, uint64_t sD2) {
  if (D > 0 && D <= 126) {
#pragma unroll
    for (int t = 0; t < N / 2; ++t) {
      float lo, hi;
      f2_unpack(f2_mul_rz_ftz(f2_pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1])), sD2), lo, hi);
      o[2 * t] = __float_as_uint(lo);
      o[2 * t + 1] = __float_as_uint(hi);
    }
  } else if (D > 126) {
    const RowRescale rr = row_rescale(D);
#pragma unroll
    for (int c = 0; c < N; ++c) o[c] = __float_as_uint(apply_rescale(__uint_as_float(o[c]), rr));
  }
}

// fl(y[c] / l) for N values of one row (l != 0, rl = the correctly rounded 1 / l), the epilogue's
// one RN division per element (reference/lssab8_golden.py:333).  When l and every y[c] lie in
// the Markstein window the N quotients are computed on pairs: each lane of the paired multiply
// and fused multiply-adds is the scalar div_markstein step (y - q l is formed as fma(q, -l, y),
// the same exact value), so the results are the correctly rounded quotients; the window test is
// a min/max of |y| over the chunk.  Otherwise each value takes div_rn_shared, after the
// contract's rescale(y, 0) (zero and subnormal -> +0) when FLUSH.
template <int N, bool FLUSH>
__device__ __forceinline__ void div_chunk(float* y, float l, float rl, bool l_in_window) {
  float mn[4], mx[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) { mn[g] = fabsf(y[g]); mx[g] = mn[g]; }
#pragma unroll
  for (int c = 4; c < N; ++c) { mn[c & 3] = fminf(mn[c & 3], fabsf(y[c])); mx[c & 3] = fmaxf(mx[c & 3], fabsf(y[c])); }
  const float lo = fminf(fminf(mn[0], mn[1]), fminf(mn[2], mn[3]));
  const float hi = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
  if (l_in_window && lo >= 0x1p-31f && hi < 0x1p32f) {
    const uint64_t rl2 = f2_pack(rl, rl), nl2 = f2_pack(-l, -l);
#pragma unroll
    for (int t = 0; t < N / 2; ++t) {
      const uint64_t y2 = f2_pack(y[2 * t], y[2 * t + 1]);
      const uint64_t q0 = f2_mul(y2, rl2);
      const uint64_t q1 = f2_fma(f2_fma(q0, nl2, y2), rl2, q0);
      f2_unpack(f2_fma(f2_fma(q1, nl2, y2), rl2, q1), y[2 * t], y[2 * t + 1]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < N; ++c) y[c] = div_rn_shared(FLUSH ? rescale(y[c], 0) : y[c], l, rl);
  }
}

// store n consecutive channels, vectorised when contiguous and aligned
template <typename OutT, int N>
__device__ __forceinline__ void store_chunk(OutT* dst, long long os3, const float* y) {
  constexpr int kPer = 16 / sizeof(OutT);
  if (os3 == 1 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int c = 0; c < N; c += kPer) {
      union { uint4 u; OutT e[kPer]; } pk;
#pragma unroll
      for (int t = 0; t < kPer; ++t) pk.e[t] = from_f32<OutT>(y[c + t]);
      *reinterpret_cast<uint4*>(dst + c) = pk.u;
    }
  } else {
#pragma unroll
    for (int c = 0; c < N; ++c) dst[c * os3] = from_f32<OutT>(y[c]);
  }
}

template <int DH, bool SINK, typename OutT, bool MULTI, bool GEN = false, bool KS = false>
__global__ void __launch_bounds__(kPrefillThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const PrefillArgs p) {
  using L = PrefillSmem<DH>;
  // Dynamic shared memory starts with T2 in 16 copies per entry (a half-warp's lanes never
  // share a bank: entry k of copy c is the 32-bit word k * 16 + c); the start of the window is a
  // link-time constant, so every gather folds the table base into its immediate offset.  The
  // 1024-byte aligned tiles follow.
  extern __shared__ uint8_t smem_raw[];
  uint32_t* s_t2 = reinterpret_cast<uint32_t*>(smem_raw);
  uint8_t* smem = smem_raw + kTabBytes + ((1024u - (smem_u32(smem_raw + kTabBytes) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);
  int8_t* v0row = reinterpret_cast<int8_t*>(smem + L::kV0);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile = p.Tpad / 128;
  const int nrounds = (ntile * p.B * p.H + (int)gridDim.x - 1) / (int)gridDim.x;

  // ---- setup, once per CTA: barriers, T2 copies, TMEM
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kBarQFull + s], 1);   mbar_init(&bars[kBarQEmpty + s], 1 + 256);
      mbar_init(&bars[kBarKFull + s], 1);   mbar_init(&bars[kBarKEmpty + s], 1);
      mbar_init(&bars[kBarVFull + s], 1);   mbar_init(&bars[kBarVEmpty + s], 1);
      mbar_init(&bars[kBarAFull + s], 1);   mbar_init(&bars[kBarAEmpty + s], 256);
      mbar_init(&bars[kBarPFull + s], 256); mbar_init(&bars[kBarPEmpty + s], 1);
    }
    mbar_init(&bars[kBarSFull], 1);
    mbar_init(&bars[kBarSEmpty], 256);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int w4 = threadIdx.x; w4 < 4096 / 16; w4 += blockDim.x)            // the A bias block
    st_shared_v4(smem_u32(smem + L::kMagic) + w4 * 16, kMagicBits, kMagicBits, kMagicBits, kMagicBits);
  fence_async_smem();                                // read by tcgen05.cp (async proxy)
  for (int k4 = threadIdx.x; k4 * 4 < kTabEntries; k4 += blockDim.x) {   // 4 entries per thread,
    const uint32_t word = (k4 * 4 < kTabLive) ? reinterpret_cast<const uint32_t*>(kT2Live)[k4] : 0u;
#pragma unroll
    for (int e = 0; e < 4; ++e) {                    // entry k -> 16 copies, 64 bytes
      const int k = k4 * 4 + e;
      if (k < kTabEntries) {
        const uint32_t t = (word >> (8 * e)) & 0xFFu;
        const uint32_t a = smem_u32(s_t2 + k * kTabCopies);
#pragma unroll
        for (int c = 0; c < kTabCopies; c += 4) st_shared_v4(a + c * 4, t, t, t, t);
      }
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= 2) {                                   // row workers: zero O
    const uint32_t rowb = tmem + ((uint32_t)((warp & 3) * 32 + ((warp - 2) >> 2) * 16) << 16);
#pragma unroll
    for (int cc = 0; cc < DH / 32; ++cc) tmem_fill16x2<DH / 2>(rowb + kColO + cc * 16, 0u);
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();                                        // the quantisers' lattice is complete

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      int jj = 0, tt = 0;
      bool ok = true;
      PfItem it;
      for (int rd = 0; ok && rd < nrounds; ++rd) {
        if (!pf_item(p, ntile, rd, it)) continue;
        const int g = it.h / p.group;
        const int qrow0 = (it.b * p.H + it.h) * p.Tpad + it.tile * 128;
        const int krow0 = (it.b * p.KVH + g) * (p.nblk * 128);
        const int qb = tt & 1;
        // buffer qb is free once item tt - 2's last QK has finished and its workers are done
        if (!mbar_wait(&bars[kBarQEmpty + qb], ((tt >> 1) & 1) ^ 1, abort_flag, p.err, 128, p.wait_ns)) { ok = false; break; }
        mbar_expect_tx(&bars[kBarQFull + qb], L::kTile + (SINK ? DH : 0));
        tma_load_2d(smem + L::kQ + qb * L::kTile, &tm_q, 0, qrow0, &bars[kBarQFull + qb]);
        if (SINK) bulk_g2s(v0row + qb * 128, p.v8 + (long long)krow0 * DH, DH, &bars[kBarQFull + qb]);
        const int nbk = (GEN && !p.causal) ? p.nblk : it.kt + 1;   // key blocks of this item
        for (int j = 0; j < nbk; ++j, ++jj) {
          const int s = jj & 1;
          const uint32_t ph = (jj >> 1) & 1;
          if (!mbar_wait(&bars[kBarKEmpty + s], ph ^ 1, abort_flag, p.err, 128, p.wait_ns)) { ok = false; break; }
          mbar_expect_tx(&bars[kBarKFull + s], L::kTile);
          // (the timeout self-test withholds one block: its bytes are expected but never arrive)
          if (tt != 0 || j != p.withhold)
            tma_load_2d(smem + L::kK + s * L::kTile, &tm_k, 0, krow0 + j * 128, &bars[kBarKFull + s]);
          if (!mbar_wait(&bars[kBarVEmpty + s], ph ^ 1, abort_flag, p.err, 128, p.wait_ns)) { ok = false; break; }
          mbar_expect_tx(&bars[kBarVFull + s], L::kTile);
          tma_load_2d(smem + L::kV + s * L::kTile, &tm_v, 0, krow0 + j * 128, &bars[kBarVFull + s]);
        }
        ++tt;
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kSwz = (DH == 128) ? 2u : 4u;          // 128B / 64B swizzle
      constexpr uint32_t kRowGroup = 8 * DH;                    // bytes per 8 rows of a tile
      constexpr uint32_t idesc_qk = idesc_i8(1, 1, 0, 128, 128);
      constexpr uint32_t idesc_pv = idesc_i8(0, 1, 1, 128, DH);
      // the bias block as a no-swizzle 128-row x 32-byte matrix: core matrices of 8 rows x 16 B,
      // 128 B apart along a row, 256 B apart down the rows (every word is the same, so only the
      // extent matters: the copy reads 4 KB)
      const uint64_t desc_bias = umma_desc(smem_u32(smem + L::kMagic), 128, 256, 0);
      int jj = 0, tt = 0;                                       // global block / item counters
      bool ok = true;
      auto issue_qk = [&](int jg, uint32_t sq) -> bool {
        const int s = jg & 1;
        const uint32_t ph = (jg >> 1) & 1;
        if (!mbar_wait(&bars[kBarKFull + s], ph, abort_flag, p.err, 0, p.wait_ns)) return false;
        // S is single-buffered: QK(jg) waits until the chain has copied S(jg - 1) into registers
        // (the jg-th phase of S_empty, jg >= 1)
        if (jg > 0 && !mbar_wait(&bars[kBarSEmpty], (jg - 1) & 1, abort_flag, p.err, 0, p.wait_ns)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + L::kK + s * L::kTile);
#pragma unroll
        for (int kk = 0; kk < DH / 32; ++kk) {
          umma_i8(tmem + kColS, umma_desc(sq + kk * 32, 16, kRowGroup, kSwz),
                  umma_desc(sk + kk * 32, 16, kRowGroup, kSwz), idesc_qk, kk > 0);
        }
        umma_commit(&bars[kBarSFull]);
        umma_commit(&bars[kBarKEmpty + s]);
        return true;
      };
      PfItem it;
      for (int rd = 0; ok && rd < nrounds; ++rd) {
        if (!pf_item(p, ntile, rd, it)) continue;
        const int nb = (GEN && !p.causal) ? p.nblk : it.kt + 1;
        const int qb = tt & 1;
        if (!mbar_wait(&bars[kBarQFull + qb], (tt >> 1) & 1, abort_flag, p.err, 0, p.wait_ns)) { ok = false; break; }
        const uint32_t sq = smem_u32(smem + L::kQ + qb * L::kTile);
        ok = issue_qk(jj, sq);
        if (ok && nb == 1) umma_commit(&bars[kBarQEmpty + qb]);   // the item's last QK is issued
        for (int j = 0; ok && j < nb; ++j) {
          const int jg = jj + j;
          if (j + 1 < nb) {
            if (!issue_qk(jg + 1, sq)) { ok = false; break; }
            if (j + 2 == nb) umma_commit(&bars[kBarQEmpty + qb]);
          }
          const int s = jg & 1;
          const uint32_t ph = (jg >> 1) & 1;
          const int sa = MULTI ? 0 : s;                             // A buffer and its use parity
          const uint32_t pha = MULTI ? (uint32_t)(jg & 1) : ph;
          if (!mbar_wait(&bars[kBarPFull + s], ph, abort_flag, p.err, 0, p.wait_ns)) { ok = false; break; }
          if (!mbar_wait(&bars[kBarVFull + s], ph, abort_flag, p.err, 0, p.wait_ns)) { ok = false; break; }
          // the fold of the block that last used this A buffer is done (jg - 2; jg - 1 in MULTI)
          if (!mbar_wait(&bars[kBarAEmpty + sa], pha ^ 1, abort_flag, p.err, 0, p.wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sp = smem_u32(smem + L::kP + s * 16384);
          const uint32_t sv = smem_u32(smem + L::kV + s * L::kTile);
#pragma unroll
          for (int c8 = 0; c8 < DH / 8; ++c8) tmem_cp_128x256b(tmem + kColA + sa * 128 + c8 * 8, desc_bias);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // A = P (K-major SW128, 32 keys = 32 bytes per step); B = V (MN-major: 32 keys =
            // 4 groups of 8 rows per step; LBO = MN-atom stride (one atom), SBO = 8-row stride).
            // Every step accumulates: the accumulator starts at the 1.5 * 2^23 bias.
            umma_i8(tmem + kColA + sa * 128, umma_desc(sp + kk * 32, 16, 1024, 2),
                    umma_desc(sv + kk * 32 * DH, L::kTile, kRowGroup, kSwz), idesc_pv, 1u);
          }
          umma_commit(&bars[kBarAFull + sa]);
          umma_commit(&bars[kBarVEmpty + s]);
          umma_commit(&bars[kBarPEmpty + s]);
        }
        jj += nb;
        ++tt;
      }
    }
  } else {
    // ================================================================ row workers
    // Warp w owns 16 query rows (TMEM lanes 32 (w % 4) + 16 ((w - 2) / 4) + [0, 16)); lanes t and
    // t + 16 of the warp share row t: lane t takes keys [0, 64) of every block's chain and
    // channels [0, DH/2) of the fold and output, lane t + 16 keys [64, 128) and channels
    // [DH/2, DH) (tcgen05.ld/st 16x32bx2 shapes).  The halves of a row meet by warp shuffles, so
    // the workers never wait on each other; every wait is on an mbarrier, per warp.
    // Iteration j runs the chain of block j, then folds block j - 1 (its A_{j-1} finished on the
    // tensor core while the chain ran).
    constexpr int HALF = DH / 2;
    const int q4 = warp & 3;
    const int row0 = q4 * 32 + ((warp - 2) >> 2) * 16;   // first TMEM lane of this warp
    const int kh = lane >> 4;                          // key half / channel half
    const int r = row0 + (lane & 15);
    const uint32_t rowt = tmem + ((uint32_t)row0 << 16);
    const uint32_t lane4 = (uint32_t)(lane & 15) << 2;
    const uint8_t* tab = reinterpret_cast<const uint8_t*>(s_t2);
    const uint32_t obase = rowt + kColO;
    const uint32_t orbase = rowt + kColOrow;             // O_row (MULTI)
    const uint64_t negM2 = f2_pack(-12582912.0f, -12582912.0f);
    const uint32_t prow = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    int jj0 = 0, tt = 0;                                 // global index of the item's block 0; item count
    bool ok = true;
    PfItem it;
    for (int rd = 0; ok && rd < nrounds; ++rd) {
      if (!pf_item(p, ntile, rd, it)) continue;
      const int tile = it.tile, kt = it.kt, b = it.b, h = it.h;
      const int g = h / p.group;
      const int nb = (GEN && !p.causal) ? p.nblk : kt + 1;   // causal: key blocks 0 .. kt
      const int qrow0 = (b * p.H + h) * p.Tpad + tile * 128;
      const int qb = tt & 1;
      const int8_t* v0 = v0row + qb * 128;               // key 0's value row of this item (sink)
      const int eqr = p.eq[(long long)qrow0 + r];
      const int32_t* ekg = p.ek + (long long)(b * p.KVH + g) * p.nblk;
      const int32_t* evg = p.ev + (long long)(b * p.KVH + g) * p.nblk;
      const int ev0 = SINK ? p.ev0[b * p.KVH + g] : 0;
      // fold state: both lanes of a row compute it identically
      float lseg = 0.0f, lrow = 0.0f;
      int nbrun = 0, nbrow = 0;
      bool have_seg = false, have_row = false;
      const bool mseg = MULTI && nb > kSEG;              // this item's rows span > 1 segment

      // fold of block jf: O = fl(O + f32(A) 2^-(s + e_v)), l = fl(l + l_b 2^-s), with the running
      // maximum rescale first (reference/lssab8_golden.py:293-315); then, at a segment end, the
      // segment -> row fold (reference/lssab8_golden.py:317-331).
      auto fold_block = [&](int jf, int nbb, int lbt, int evj, int eh0v, bool live) -> bool {
        const int jgf = jj0 + jf;                          // global block index (pipeline parities)
        const int sa = MULTI ? 0 : (jgf & 1);
        const uint32_t pha = MULTI ? (uint32_t)(jgf & 1) : (uint32_t)((jgf >> 1) & 1);
        int sg = 0, Dr = 0;
        if (!GEN || live) {
          if (!have_seg) { nbrun = nbb; have_seg = true; }
          const int D = nbb - nbrun;
          if (D > 0) { Dr = D; lseg = rescale(lseg, D); nbrun = nbb; }
          else sg = -D;
        } else {
          sg = kSWIN + 1;                                  // a hidden block: no update, a zero term
        }
        if (!warp_poll(&bars[kBarAFull + sa], pha, abort_flag, p.err, p.wait_ns)) return false;
        // key 0's value row arrives with the item's Q tile
        if (SINK && jf == 0 && p.T > 1 && !warp_poll(&bars[kBarQFull + qb], (tt >> 1) & 1, abort_flag, p.err, p.wait_ns)) return false;
        tc_fence_after();
        // A block beyond the exact-skip window (sg > S_WIN) is folded with scale +0 instead of being
        // skipped: O and l are never -0 (they start at +0, an RN sum that cancels exactly is +0, and
        // the rescale flushes to +0), and A_b, l_b are finite, so O + (+0) x == O bit for bit.
        const bool add = (sg <= kSWIN);
        const float scO = add ? pow2f(-(sg + evj)) : 0.0f;
        const uint64_t scO2 = f2_pack(scO, scO);
        const bool resc = __any_sync(0xffffffffu, Dr > 0);  // warp-uniform
        // rows with D > 0 have sg == 0, so the term added after their rescale has the positive
        // scale 2^-e_v (|e_v| <= 126 for finite inputs) and turns a flushed -0 into +0
        const uint64_t sD2 = f2_pack(pow2f(-min(Dr, 126)), pow2f(-min(Dr, 126)));
        // DH/2 channels per lane in passes of 32 (two TMEM round trips for DH = 128); the next
        // pass's loads are issued before this pass's stores, so their latency overlaps
        constexpr int kPass = HALF < 32 ? HALF : 32;
        constexpr int kNPass = HALF / kPass;
        const uint32_t abase = rowt + kColA + sa * 128;
        auto fold_pass = [&](int c0, uint32_t* a, uint32_t* o) {
          if (resc) rescale_channels<kPass>(o, Dr, sD2);
          if (SINK && jf == 0 && p.T > 1) {                  // key 0's term first (B9.1); sg == 0 here
            const float sc0 = pow2f(-ev0);
            const uint64_t sc02 = f2_pack(sc0, sc0);
  #pragma unroll
            for (int t = 0; t < kPass / 2; ++t) {
              const int c = kh * HALF + c0 + 2 * t;
              const uint64_t z = f2_pack(i2f_small(eh0v * (int)v0[c]), i2f_small(eh0v * (int)v0[c + 1]));
              float lo_, hi_;
              f2_unpack(f2_fma(z, sc02, f2_pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1]))), lo_, hi_);
              o[2 * t] = __float_as_uint(lo_);
              o[2 * t + 1] = __float_as_uint(hi_);
            }
          }
  #pragma unroll
          for (int t = 0; t < kPass / 2; ++t) {
            const uint64_t x = f2_add(f2_pack(__uint_as_float(a[2 * t]), __uint_as_float(a[2 * t + 1])), negM2);
            float lo_, hi_;
            f2_unpack(f2_fma(x, scO2, f2_pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1]))), lo_, hi_);
            o[2 * t] = __float_as_uint(lo_);
            o[2 * t + 1] = __float_as_uint(hi_);
          }
        };
        auto load_pass = [&](int c0, uint32_t* a, uint32_t* o) {
  #pragma unroll
          for (int cc = 0; cc < kPass / 16; ++cc) {
            tmem_ld16x2<HALF>(abase + c0 + cc * 16, a + cc * 16);
            tmem_ld16x2<HALF>(obase + c0 + cc * 16, o + cc * 16);
          }
        };
        auto store_pass = [&](int c0, const uint32_t* o) {
  #pragma unroll
          for (int cc = 0; cc < kPass / 16; ++cc) tmem_st16x2<HALF>(obase + c0 + cc * 16, o + cc * 16);
        };
        {
          uint32_t a0[kPass], o0[kPass];
          load_pass(0, a0, o0);
          tc_wait_ld();
          fold_pass(0, a0, o0);
          if constexpr (kNPass == 2) {
            uint32_t a1[kPass], o1[kPass];
            load_pass(kPass, a1, o1);
            store_pass(0, o0);
            tc_wait_ld();
            fold_pass(kPass, a1, o1);
            store_pass(kPass, o1);
          } else {
            store_pass(0, o0);
          }
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[kBarAEmpty + sa]);
        lseg = fold_term(lseg, lbt, add ? pow2f(-sg) : 0.0f);
        if (mseg && (((jf + 1) % kSEG == 0) || (jf == nb - 1))) {
          // segment -> row: the same three rules (reference/lssab8_golden.py:317-331), TMEM to
          // TMEM; first, D2 and s2 are per row and stay in the arithmetic (the TMEM accesses are
          // the warp's, unconditional); a row whose segment saw no key keeps its O_row (GEN)
          int D2 = 0, s2 = 0;
          const bool segl = !GEN || have_seg;
          const bool first = !have_row;
          if (segl) {
            if (first) { nbrow = nbrun; have_row = true; }
            else { D2 = nbrun - nbrow; if (D2 > 0) { lrow = rescale(lrow, D2); nbrow = nbrun; } else { s2 = -D2; } }
          }
  #pragma unroll 1
          for (int cc = 0; cc < HALF / 16; ++cc) {
            uint32_t y[16], x[16];
            tmem_ld16x2<HALF>(obase + cc * 16, y);
            tmem_ld16x2<HALF>(orbase + cc * 16, x);
            tc_wait_ld();
  #pragma unroll
            for (int c = 0; c < 16; ++c) {
              const float seg = __uint_as_float(y[c]);
              float xr = __uint_as_float(x[c]);
              if (!segl) { /* unchanged */ }
              else if (first) xr = rescale(seg, 0);
              else {
                if (D2 > 0) xr = rescale(xr, D2);
                if (s2 <= kSWIN) xr = __fadd_rn(xr, rescale(seg, s2));
              }
              x[c] = __float_as_uint(xr);
            }
            tmem_st16x2<HALF>(orbase + cc * 16, x);
            tmem_fill16x2<HALF>(obase + cc * 16, 0u);      // O_seg starts at +0 for the next segment
          }
          tc_wait_st();
          if (segl) {
            if (first) lrow = rescale(lseg, 0);
            else if (s2 <= kSWIN) lrow = __fadd_rn(lrow, rescale(lseg, s2));
          }
          lseg = 0.0f;
          have_seg = false;
        }
        return true;
      };

      int nb_prev = 0, ev_prev = 0, lbt_prev = 0, eh0_row = 0;
      bool live_prev = true;
      int ek_next = ekg[0], ev_next = evg[0];            // e_k, e_v one block ahead
      // GEN: this lane's 64 key-mask bits, one block ahead
      const uint32_t* kmb = GEN ? p.kmask + (long long)b * p.nblk * 4 + kh * 2 : nullptr;
      uint2 km_next = GEN ? make_uint2(kmb[0], kmb[1]) : make_uint2(0u, 0u);
      // KS: this lane's 64 weight shifts (one byte per key), one block ahead
      const uint4* dsb = KS ? reinterpret_cast<const uint4*>(p.d8 + (long long)(b * p.KVH + g) * p.nblk * 128 + kh * 64)
                            : nullptr;
      uint4 ds_next[4], ds_cur[4];
      if (KS) {
  #pragma unroll
        for (int i = 0; i < 4; ++i) ds_next[i] = dsb[i];
      }
      for (int j = 0; j < nb; ++j) {
        const int ekj = ek_next, evj = ev_next;
        const uint2 kmj = km_next;
        if (KS) {
  #pragma unroll
          for (int i = 0; i < 4; ++i) ds_cur[i] = ds_next[i];
        }
        if (j + 1 < nb) {
          ek_next = ekg[j + 1]; ev_next = evg[j + 1];
          if (GEN) km_next = make_uint2(kmb[(j + 1) * 4], kmb[(j + 1) * 4 + 1]);
          if (KS) {
  #pragma unroll
            for (int i = 0; i < 4; ++i) ds_next[i] = dsb[(j + 1) * 8 + i];   // 128 keys = 8 x 16 bytes
          }
        }
        const int jg = jj0 + j;
        const int s = jg & 1;
        const uint32_t ph = (jg >> 1) & 1;
        // G and the exact-window width need only the exponents: computed while S(j) is in flight
        const uint32_t G = g_fold(p.gbase, eqr + ekj);
        const int lg = 31 - __clz((int)G);
        const int dm = 1 << max(0, 30 - lg);              // dm * G in [2^30, 2^31): >= 9 doublings
        const uint32_t negG = 0u - G;
        // P buffer s is free once PV(j - 2) has finished -- long before S(j) is ready
        if (!warp_poll(&bars[kBarPEmpty + s], ph ^ 1, abort_flag, p.err, p.wait_ns)) { ok = false; break; }
        if (!warp_poll(&bars[kBarSFull], jg & 1, abort_flag, p.err, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
        const bool diag = (j == kt) && (!GEN || p.causal);  // key c of the diagonal block visible iff c <= r
        // pass 1: this lane's 64 scores into registers (one TMEM round trip; S is free for the
        // next QK as soon as they have landed) and the exact max over its visible keys
        uint32_t v[64];
        const uint32_t sbase = rowt + kColS;
        tmem_ld16x2<64>(sbase, v);
        tmem_ld16x2<64>(sbase + 16, v + 16);
        tmem_ld16x2<64>(sbase + 32, v + 32);
        tmem_ld16x2<64>(sbase + 48, v + 48);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[kBarSEmpty]);
        if (diag) {
  #pragma unroll
          for (int c = 0; c < 64; ++c) if (kh * 64 + c > r) v[c] = 0x80000000u;
        }
        if (GEN) {                                         // hidden keys
  #pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (!((kmj.x >> c) & 1u)) v[c] = 0x80000000u;
            if (!((kmj.y >> c) & 1u)) v[32 + c] = 0x80000000u;
          }
        }
        // four independent 16-score maxima, then their maximum: a dependency depth of 9 instead of 32
        int mq[4];
  #pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          const uint32_t* vg = v + 16 * g4;
          int a = __vimax3_s32((int)vg[0], (int)vg[1], (int)vg[2]);
  #pragma unroll
          for (int c = 3; c < 15; c += 2) a = __vimax3_s32(a, (int)vg[c], (int)vg[c + 1]);
          mq[g4] = max(a, (int)vg[15]);
        }
        int m = max(__vimax3_s32(mq[0], mq[1], mq[2]), mq[3]);
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 16));  // the row's max over both key halves
        // a row that sees no key of this block (GEN) gets an all-zero weight row: with m = 0 and
        // NB = 0 every hidden key's d = dm G >= 2^30 lands past the table's live range
        const bool live = !GEN || (m != (int)0x80000000);
        if (GEN && !live) m = 0;
        const int nbv = nb_of(m, G);
        const uint32_t NBlo = (uint32_t)nbv << kBHI;
        const int lo = m - dm;
        const uint32_t pbase = smem_u32(smem + L::kP + s * 16384) + prow;
        uint32_t lbq[2] = {0u, 0u}, eh0 = 0;               // two l_b partial sums (shorter dp4a chains)
        // pass 2: the chain and the u8 P half-row, 16 keys (one 16-byte P chunk) at a time
  #pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t w[4];
  #pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            uint32_t e[4];
  #pragma unroll
            for (int x = 0; x < 4; ++x) {
              const int sc = max((int)v[cc * 16 + qq * 4 + x], lo);
              uint32_t d = NBlo + (uint32_t)sc * negG;       // exact: d < 2^32
              const uint32_t ix = min(d, kDClamp) >> kIdxShift;  // index <= 1152 (T2 = 0 from 1152 on)
              e[x] = tab[ix * p.mul_entry + lane4];            // entry ix, this lane's copy
            }
            w[qq] = e[0] + e[1] * p.mul_b1 + e[2] * p.mul_b2 + e[3] * p.mul_b3;
            lbq[qq & 1] = __dp4a(w[qq], 0x01010101u, lbq[qq & 1]);   // l_b: the unshifted weights
            if (KS) {                                        // the PV weights eh >> d
              const uint32_t dw = qq == 0 ? ds_cur[cc].x : qq == 1 ? ds_cur[cc].y : qq == 2 ? ds_cur[cc].z : ds_cur[cc].w;
              w[qq] = (e[0] >> (dw & 0xFFu)) | ((e[1] >> ((dw >> 8) & 0xFFu)) << 8) |
                      ((e[2] >> ((dw >> 16) & 0xFFu)) << 16) | ((e[3] >> (dw >> 24)) << 24);
            }
          }
          const int chunk = kh * 4 + cc;
          if (SINK && chunk == 0 && j == 0 && p.T > 1) { eh0 = w[0] & 0xFFu; w[0] &= ~0xFFu; }
          st_shared_v4(pbase + (uint32_t)((chunk ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();
        mbar_arrive(&bars[kBarPFull + s]);
        const uint32_t lb = lbq[0] + lbq[1];
        const int lbt = (int)lb + __shfl_xor_sync(0xffffffffu, (int)lb, 16);   // the row's l_b
        if (SINK && j == 0) eh0_row = __shfl_sync(0xffffffffu, (int)eh0, lane & 15);
        if (j > 0 && !fold_block(j - 1, nb_prev, lbt_prev, ev_prev, eh0_row, live_prev)) { ok = false; break; }
        nb_prev = nbv;
        lbt_prev = lbt;
        ev_prev = evj;
        live_prev = live;
      }
      if (ok) ok = fold_block(nb - 1, nb_prev, lbt_prev, ev_prev, eh0_row, live_prev);

      // ---- epilogue: out = O_row / l_row (one RN division per element; l_row == 0 -> 0).
      // `ok` is warp-uniform (every wait is decided for the whole warp), so the warp-collective
      // TMEM loads run on every lane or on none; rows past T skip only the store.
      if (ok) {
        if (!mseg) lrow = rescale(lseg, 0);             // a single segment: O_row = 0 + rescale(O_seg, 0)
        const int i = kt * 128 + r;                      // the row's position in the sequence
        const bool live = (i < p.T);
        const bool nz = (lrow != 0.0f);
        const float rl = nz ? __frcp_rn(lrow) : 0.0f;
        const bool row_fast = div_window(lrow);
        OutT* dst = reinterpret_cast<OutT*>(p.out) + b * p.os0 + (long long)(i - p.tile0 * 128) * p.os1 + h * p.os2 +
                    kh * HALF * p.os3;                   // out holds the chunk's rows
  #pragma unroll 1
        for (int cc = 0; cc < HALF / 16; ++cc) {
          float q[16];
          uint32_t y[16];
          tmem_ld16x2<HALF>((mseg ? orbase : obase) + cc * 16, y);
          tc_wait_ld();
          if (!mseg) tmem_fill16x2<HALF>(obase + cc * 16, 0u);   // O starts at +0 for the next item
  #pragma unroll
          for (int c = 0; c < 16; ++c) q[c] = __uint_as_float(y[c]);
          if (live) {
            // a single segment divides rescale(O_seg, 0) (identity on the Markstein window);
            // O_row is already flushed by the segment -> row fold
            if (nz) {
              if (mseg) div_chunk<16, false>(q, lrow, rl, row_fast);
              else div_chunk<16, true>(q, lrow, rl, row_fast);
            } else {
  #pragma unroll
              for (int c = 0; c < 16; ++c) q[c] = 0.0f;
            }
            store_chunk<OutT, 16>(dst + cc * 16 * p.os3, p.os3, q);
            for (int pr = 0; pr < p.npeers; ++pr) {      // the gather: the same rows into every peer
              OutT* pd = reinterpret_cast<OutT*>(p.peers[pr]) + (dst - reinterpret_cast<OutT*>(p.out));
              store_chunk<OutT, 16>(pd + cc * 16 * p.os3, p.os3, q);
            }
          }
        }
        tc_wait_st();
      }
      // this item is done with O, its sink row and (through the MMA's commit) its Q tile
      tc_fence_before();
      mbar_arrive(&bars[kBarQEmpty + qb]);
      jj0 += nb;
      ++tt;
    }                                                  // items
  }

  // ---- teardown
  // stores into peers' memory are visible system-wide before this CTA ends, hence before the
  // kernel completes and before whatever the stream orders after it (the ranks' barrier)
  if (p.npeers > 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace lssab8
