// LSSA-B8 split-KV decode on sm_100a, tensor-core form (dh = 128).
//
// Same contract and workspace as decode_kernel (decode.cuh): every 128-key block of a sequence
// yields EXACT integer block partials (A_b = eh . v8 per head and channel, NB_b, l_b, eh0), and
// a refold folds all blocks of a (sequence, kv head) in ascending order
// (reference/lssab8_golden.py:350-394).  What changes is how the partials are produced and refolded:
//
//   * persistent CTAs walk the list of LIVE (sequence, kv head, block) triples -- numbered by a
//     per-sequence prefix sum of block counts (decode_plan_kernel), so ragged lengths leave no
//     dead work to skip and every CTA gets an even share -- in interleaved chunks of kDecChunk
//     blocks as ONE stream (block partials are exact, so where a split or chunk ends changes no
//     bit): the TMA ring never drains, the one-block lag of the partial readout runs across chunk
//     boundaries, and Q is reloaded only when (sequence, kv head) changes;
//   * warp 0 (one thread) streams each block's 8 key pages with cp.async.bulk.tensor (the tensor
//     map swizzles them into the SW128 K-major layout) and its 8 transposed value pages with
//     plain cp.async.bulk into a kDecStages-deep ring (no multicast);
//   * warp 1 (one thread) owns 64 TMEM columns and issues both contractions on the tensor core,
//     kind::i8 with the GQA group padded to N = 16:
//       S^T[key, head] = K_b[128 x 128] . Q^T     (s8 x s8, both K-major SW128)
//       A^T[ch, head]  = V_b^T[128 x 128] . P^T   (s8 x u8; a value page [ch][16 keys] is exactly
//                                                  8-row x 16-byte core matrices, so V^T is read
//                                                  in place with no swizzle: LBO = one page)
//   * worker warpgroups (128 threads each, thread = TMEM lane = key for S, channel for A; one
//     warpgroup for a group of <= 4 heads, two -- heads 0-3 and 4-7 -- for a group of 8, so the
//     per-block path does not lengthen with the group) compute the block max per head (redux.sync
//     + one named barrier per warpgroup), NB, the 32-bit chain and the T2 gather from a
//     zero-padded table indexed by d >> 19, write P^T in the core-matrix layout, sum l_b with
//     redux.sync and shared atomics, and store the partials.
//   * the refold of each (sequence, kv head, head) runs afterwards as its own small kernel
//     (decode_merge_kernel), longest sequences first, so no streaming CTA ever stalls on a merge.
#pragma once
#include "decode.cuh"

namespace lssab8 {

constexpr int kDecStages = 3;                      // two CTAs per SM, three stages each
constexpr int kDecTab = 1168;                      // T2 entries 0..1152 (1152 = 0), 16-byte padded
// warp 0 TMA, warp 1 MMA + TMEM, then one worker warpgroup per 4 heads of the group
template <int GQ> struct DecWorkers {
  static constexpr int kGroups = GQ > 4 ? 2 : 1;     // warpgroups
  static constexpr int kHeads = GQ / kGroups;        // heads per warpgroup (4)
  static constexpr int kThreads = 64 + 128 * kGroups;
};
constexpr uint32_t kDecTmemCols = 64;

struct DecTcSmem {
  static constexpr int kPage = 16 * 128;                  // one page of one kv head (dh 128), bytes
  static constexpr int kStage = 16 * kPage;               // 8 key pages, then 8 value pages
  static constexpr int kQ = kDecStages * kStage;          // 2 x Q^T [16 rows x 128 B], SW128
  static constexpr int kP = kQ + 2 * 2048;                // 2 x P^T [16 heads x 128 keys], core matrices
  static constexpr int kTab = kP + 2 * 2048;              // T2 entries 0..1152 (index clamped to 1152)
  static constexpr int kRedMax = kTab + kDecTab;          // [2][4 warps][8 heads] block max
  static constexpr int kLbSum = kRedMax + 2 * 4 * 8 * 4;  // [2][8] l_b
  static constexpr int kNb = kLbSum + 2 * 8 * 4;          // [2][8] NB_b
  static constexpr int kEh0 = kNb + 2 * 8 * 4;            // [2][8] key 0's weight (sink, block 0)
  static constexpr int kBar = kEh0 + 2 * 8 * 4 + 32;      // mbarriers
  static constexpr int kMisc = kBar + 32 * 8;             // tmem base, abort flag
  static constexpr int kBytes = kMisc + 64;
};

enum DecBar : int {
  kDFull = 0, kDEmpty = kDecStages, kDQFull = 2 * kDecStages, kDQEmpty = kDQFull + 2, kDSFull = kDQEmpty + 2,
  kDSEmpty = kDSFull + 2, kDPFull = kDSEmpty + 2, kDPEmpty = kDPFull + 2, kDAFull = kDPEmpty + 2,
  kDAEmpty = kDAFull + 2, kDNumBars = kDAEmpty + 2
};

constexpr int kDecChunk = 8;                       // blocks per scheduling chunk

// The CTA's walk over the live block list: v = KVH * off[b] + g * nblk_b + blk for blk < nblk_b
// (off = the plan's prefix sum of live block counts, nblk_b = off[b + 1] - off[b]), in chunks of
// kDecChunk: chunks blockIdx.x, blockIdx.x + gridDim.x, ...  A CTA's v only grows, so the
// sequence of v is found by advancing one cursor over off (each CTA reads off once).  Sequences
// the plan found too long for the lattice arrays have no live blocks (and are flagged there).
// Every role runs its own copy and sees the same sequence of blocks.
struct DecIter {
  int v, vend, chunk, nchunks, total;
  int cur_b, lo, hi, nb, L;                        // this sequence's live range [lo, hi) of v
  __device__ __forceinline__ void init(const DecodeArgs& p) {
    total = p.KVH * __ldg(&p.blk_off[p.B]);
    nchunks = (total + kDecChunk - 1) / kDecChunk;
    chunk = blockIdx.x;
    v = chunk * kDecChunk;
    vend = min(v + kDecChunk, total);
    cur_b = 0;
    lo = 0;
    nb = __ldg(&p.blk_off[1]);
    hi = p.KVH * nb;
    L = __ldg(&p.seq_lens[0]);
  }
  __device__ __forceinline__ bool next(const DecodeArgs& p, int& b, int& g, int& blk) {
    if (v >= vend) {
      chunk += gridDim.x;
      if (chunk >= nchunks) return false;
      v = chunk * kDecChunk;
      vend = min(v + kDecChunk, total);
    }
    while (v >= hi) {                              // v < total, so some later sequence holds it
      ++cur_b;
      lo = hi;
      nb = __ldg(&p.blk_off[cur_b + 1]) - __ldg(&p.blk_off[cur_b]);
      hi = lo + p.KVH * nb;
      L = __ldg(&p.seq_lens[cur_b]);
    }
    const int r = v++ - lo;
    b = cur_b;
    g = r / nb;
    blk = r - g * nb;
    return true;
  }
};

// The live-block plan: blk_off[b] = the number of live 128-key blocks of the sequences before b
// (blk_off[B] = all of them), one CTA, which also zeroes the refold's tickets[0 .. nticket).  A
// sequence is live when 0 < L and its blocks and pages fit the lattice arrays; one that does not
// fit gets no blocks and sets kDevBadPage.
constexpr int kPlanThreads = 1024;
constexpr int kPlanSortMax = 1024;                 // batches up to this size get the longest-first order
__global__ void __launch_bounds__(kPlanThreads) decode_plan_kernel(const int32_t* seq_lens, int B, int max_blocks,
                                                                    int max_pages, int* blk_off, int* order,
                                                                    unsigned int* tickets, int nticket, int* err) {
  __shared__ int warp_sums[kPlanThreads / 32];
  __shared__ int carry;
  __shared__ int sl[kPlanSortMax];
  pdl_launch_dependents();                         // the query quantiser runs beside the plan
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int i = tid; i < nticket; i += kPlanThreads) tickets[i] = 0u;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < B; base += kPlanThreads) {
    const int i = base + tid;
    int nb = 0;
    if (i < B) {
      const int L = seq_lens[i];
      nb = L > 0 ? (L + kKB - 1) / kKB : 0;
      if (nb > max_blocks || (L + 15) / 16 > max_pages) {
        nb = 0;
        atomicOr(err, kDevBadPage);
      }
    }
    int x = nb;                                    // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[w] = x;
    __syncthreads();
    if (w == 0) {
      int ws = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, ws, o);
        if (lane >= o) ws += y;
      }
      warp_sums[lane] = ws;                        // inclusive over warps
    }
    __syncthreads();
    const int before = carry + (w > 0 ? warp_sums[w - 1] : 0) + x - nb;
    if (i < B) blk_off[i] = before;
    __syncthreads();
    if (tid == 0) carry += warp_sums[kPlanThreads / 32 - 1];
    __syncthreads();
  }
  // the refold's sequence order, longest first (ties by index): order[rank(i)] = i with
  // rank(i) = #{j : L_j > L_i, or L_j == L_i and j < i}; larger batches keep the index order
  if (B <= kPlanSortMax) {
    for (int i = tid; i < B; i += kPlanThreads) sl[i] = seq_lens[i];
    __syncthreads();
    for (int i = tid; i < B; i += kPlanThreads) {
      const int Li = sl[i];
      int r = 0;
      for (int j = 0; j < B; ++j) r += (sl[j] > Li || (sl[j] == Li && j < i)) ? 1 : 0;
      order[r] = i;
    }
  } else {
    for (int i = tid; i < B; i += kPlanThreads) order[i] = i;
  }
  if (tid == 0) blk_off[B] = carry;
}

__device__ __forceinline__ uint32_t redux_max_s32(int v) {
  int r;
  asm volatile("redux.sync.max.s32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return (uint32_t)r;
}
__device__ __forceinline__ uint32_t redux_add_u32(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.add.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

// GQ = compile-time bound on the GQA group (4: exactly 4 heads; 8: any group <= 8, masked).
template <bool SINK, typename OutT, int GQ>
__global__ void __launch_bounds__(DecWorkers<GQ>::kThreads, 2)
decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                 const DecodeArgs p) {
  using L = DecTcSmem;
  using WK = DecWorkers<GQ>;
  constexpr int DH = 128;
  constexpr int kWorkers = 128 * WK::kGroups;
  constexpr int GH = WK::kHeads;                       // heads per worker warpgroup
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint8_t* tab = smem + L::kTab;
  int* redmax = reinterpret_cast<int*>(smem + L::kRedMax);
  uint32_t* lbsum = reinterpret_cast<uint32_t*>(smem + L::kLbSum);
  int* nbs = reinterpret_cast<int*>(smem + L::kNb);
  int* eh0s = reinterpret_cast<int*>(smem + L::kEh0);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = p.group;

  for (int i = threadIdx.x; i < kDecTab; i += blockDim.x) tab[i] = (i < kTabLive) ? kT2Live[i] : 0;
  for (int i = threadIdx.x; i < 2 * 8; i += blockDim.x) lbsum[i] = 0u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) { mbar_init(&bars[kDFull + s], 1); mbar_init(&bars[kDEmpty + s], 1); }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kDQFull + s], 1);  mbar_init(&bars[kDQEmpty + s], 1);
      mbar_init(&bars[kDSFull + s], 1);  mbar_init(&bars[kDSEmpty + s], kWorkers);
      mbar_init(&bars[kDPFull + s], kWorkers); mbar_init(&bars[kDPEmpty + s], 1);
      mbar_init(&bars[kDAFull + s], 1);  mbar_init(&bars[kDAEmpty + s], kWorkers);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kDecTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();                             // the refold kernel may queue up behind us
  pdl_wait();                                          // the plan and the query quantiser are complete

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      DecIter itr;
      itr.init(p);
      int jj = 0, run = -1, cur_bg = -1, b, g, blk;
      const uint64_t once = l2_evict_first_policy();    // the lattice is read once per call
      while (itr.next(p, b, g, blk)) {
        const int bg = b * p.KVH + g;
        if (bg != cur_bg) {                              // a new (sequence, kv head): its Q^T tile
          cur_bg = bg;
          ++run;
          const int qb = run & 1;
          if (!mbar_wait(&bars[kDQEmpty + qb], ((run >> 1) & 1) ^ 1, abort_flag, p.err, 128)) break;
          mbar_expect_tx(&bars[kDQFull + qb], 2048);
          tma_load_2d(smem + L::kQ + qb * 2048, &tm_q, 0, b * p.H + g * gq, &bars[kDQFull + qb]);
        }
        const int st = jj % kDecStages;
        const int npg = min(8, (itr.L - blk * kKB + 15) / 16);
        const int32_t* bt = p.block_table + (long long)b * p.max_pages + blk * 8;
        int pg[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pg[i] = (i < npg) ? bt[i] : 0;   // in flight during the wait
        if (!mbar_wait(&bars[kDEmpty + st], ((jj / kDecStages) & 1) ^ 1, abort_flag, p.err, 128)) break;
        mbar_expect_tx(&bars[kDFull + st], (uint32_t)(npg * 2 * L::kPage));
        uint8_t* kdst = smem + st * L::kStage;
        uint8_t* vdst = kdst + 8 * L::kPage;
        for (int i = 0; i < npg; ++i) {
          int q = pg[i];
          if (q < 0 || q >= p.num_pages) { atomicOr(p.err, kDevBadPage); q = 0; }
          const long long prow = (long long)q * p.KVH + g;
          tma_load_2d_hint(kdst + i * L::kPage, &tm_k, 0, (int)(prow * 16), &bars[kDFull + st], once);
          bulk_g2s_hint(vdst + i * L::kPage, p.v8p + prow * L::kPage, L::kPage, &bars[kDFull + st], once);
        }
        ++jj;
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_i8(1, 1, 0, 128, 16);
      constexpr uint32_t idesc_pv = idesc_i8(1, 0, 0, 128, 16);
      auto issue_pv = [&](int jb) -> bool {
        const int ab = jb & 1, st = jb % kDecStages;
        if (!mbar_poll(&bars[kDPFull + ab], (jb >> 1) & 1, abort_flag, p.err)) return false;
        if (!mbar_poll(&bars[kDAEmpty + ab], ((jb >> 1) & 1) ^ 1, abort_flag, p.err)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + st * L::kStage + 8 * L::kPage);
        const uint32_t sp = smem_u32(smem + L::kP + ab * 2048);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // 32 keys = 2 pages (A) / 2 core matrices (B) per step
          umma_i8(tmem + 32 + ab * 16, umma_desc(sv + kk * 2 * L::kPage, L::kPage, 128, 0),
                  umma_desc(sp + kk * 2 * 256, 256, 128, 0), idesc_pv, kk > 0);
        umma_commit(&bars[kDAFull + ab]);
        umma_commit(&bars[kDEmpty + st]);
        umma_commit(&bars[kDPEmpty + ab]);
        return true;
      };
      DecIter itr;
      itr.init(p);
      int jj = 0, run = -1, cur_bg = -1, b, g, blk;
      bool ok = true;
      while (ok && itr.next(p, b, g, blk)) {
        const int bg = b * p.KVH + g;
        if (bg != cur_bg) {
          // every QK of the previous (sequence, kv head) is issued: its Q^T buffer frees when they finish
          if (run >= 0) umma_commit(&bars[kDQEmpty + (run & 1)]);
          cur_bg = bg;
          ++run;
          if (!mbar_poll(&bars[kDQFull + (run & 1)], (run >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
        }
        const uint32_t sq = smem_u32(smem + L::kQ + (run & 1) * 2048);
        const int st = jj % kDecStages, sb = jj & 1;
        if (!mbar_poll(&bars[kDFull + st], (jj / kDecStages) & 1, abort_flag, p.err)) { ok = false; break; }
        if (!mbar_poll(&bars[kDSEmpty + sb], ((jj >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + st * L::kStage);
#pragma unroll
        for (int kk = 0; kk < DH / 32; ++kk)
          umma_i8(tmem + sb * 16, umma_desc(sk + kk * 32, 16, 1024, 2), umma_desc(sq + kk * 32, 16, 1024, 2),
                  idesc_qk, kk > 0);
        umma_commit(&bars[kDSFull + sb]);
        if (jj > 0 && !issue_pv(jj - 1)) { ok = false; break; }   // PV lags QK by one block
        ++jj;
      }
      if (ok && jj > 0) issue_pv(jj - 1);
    }
  } else {
    // ================================================================ workers
    // Warpgroup wg (warps 2 + 4 wg .. 5 + 4 wg) owns heads [wg * GH, wg * GH + GH) of the group;
    // thread t of a warpgroup is TMEM lane t: key t of S, channel t of A.  The warpgroups meet
    // only on the pipeline barriers (which count every worker thread), never on each other.
    const int wg = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int t = wq * 32 + lane;                        // TMEM lane: key (S) / channel (A)
    const int h0 = wg * GH;                              // first head of this warpgroup
    const int bar_id = 1 + wg;                           // this warpgroup's named barrier
    const uint32_t lanebase = tmem + ((uint32_t)(wq * 32) << 16);
    DecIter itr;
    itr.init(p);
    int jj = 0, cur_bg = -1, b, g, blk;
    bool bad = false;                                    // this warp gave up a wait (decided at a barrier)
    int eqh[GH];
    // the previous block: its A partial is read out one block later, its M after the next barrier
    bool have_prev = false;
    long long prev_bg = 0;
    int prev_blk = 0, prev_L = 0;
    auto readout_A = [&](int jb, long long bgx, int blkx) -> bool {
      const int ab = jb & 1;
      const bool okw = warp_poll(&bars[kDAFull + ab], (jb >> 1) & 1, abort_flag, p.err);
      if (okw) {
        tc_fence_after();
        uint32_t a[GH];
        tmem_ld4(lanebase + 32 + ab * 16 + h0, a);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[kDAEmpty + ab]);
        int32_t* dstA = p.partA + ((bgx * p.max_blocks + blkx) * gq) * DH;
#pragma unroll
        for (int hh = 0; hh < GH; ++hh) if (h0 + hh < gq) __stcg(dstA + (h0 + hh) * DH + t, (int32_t)a[hh]);
      }
      return okw;
    };
    auto write_M = [&](int jb, long long bgx, int blkx, int Lx) {   // after a barrier that follows jb's atomics
      const int par = jb & 1;
      const int h = h0 + t;
      if (t < GH && h < gq) {
        const int e0 = (SINK && blkx == 0 && Lx > 1) ? eh0s[par * 8 + h] : 0;
        __stcg(&p.partM[(bgx * p.max_blocks + blkx) * gq + h], make_int4(nbs[par * 8 + h], (int)lbsum[par * 8 + h], e0, 0));
        lbsum[par * 8 + h] = 0u;
      }
    };
    while (itr.next(p, b, g, blk)) {
      const long long bg = (long long)b * p.KVH + g;
      if (bg != cur_bg) {
        cur_bg = bg;
#pragma unroll
        for (int hh = 0; hh < GH; ++hh) eqh[hh] = (h0 + hh < gq) ? p.eq[(long long)b * p.H + g * gq + h0 + hh] : 0;
      }
      const int Lb = itr.L;
      const int sb = jj & 1, par = jj & 1;
      const int ekb = p.ek[bg * p.max_blocks + blk];
      bool okw = warp_poll(&bars[kDSFull + sb], (jj >> 1) & 1, abort_flag, p.err);
      int S[GH];
      if (okw) {
        tc_fence_after();
        tmem_ld4(lanebase + sb * 16 + h0, reinterpret_cast<uint32_t*>(S));
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[kDSEmpty + sb]);
      }
      const int nkeys = min(kKB, Lb - blk * kKB);
      if (t >= nkeys) {
#pragma unroll
        for (int hh = 0; hh < GH; ++hh) S[hh] = INT32_MIN;  // keys past the sequence end
      }
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        const int wm = (int)redux_max_s32(S[hh]);
        if (lane == 0) redmax[(par * 4 + wq) * 8 + h0 + hh] = wm;
      }
      uint32_t Gh[GH];
      int dmh[GH];
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {                  // independent of the block max: before the barrier
        Gh[hh] = g_fold(p.gbase, eqh[hh] + ekb);
        dmh[hh] = 1 << max(0, 30 - (31 - __clz((int)Gh[hh])));
      }
      // the warpgroup meets here once per block; the OR makes giving up a group decision
      if (bar_any(bar_id, 128, bad || !okw || *abort_flag != 0)) { have_prev = false; break; }
      if (have_prev) write_M(jj - 1, prev_bg, prev_blk, prev_L);   // the previous block's l_b atomics are complete
      uint32_t e[GH];
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        const int h = h0 + hh;
        const int m = max(max(redmax[(par * 4 + 0) * 8 + h], redmax[(par * 4 + 1) * 8 + h]),
                          max(redmax[(par * 4 + 2) * 8 + h], redmax[(par * 4 + 3) * 8 + h]));
        const uint32_t G = Gh[hh];
        const int nbv = nb_of(m, G);
        const int sc = max(S[hh], m - dmh[hh]);
        const uint32_t d = ((uint32_t)nbv << kBHI) + (uint32_t)sc * (0u - G);
        e[hh] = (h < gq && t < nkeys) ? (uint32_t)tab[min(d >> kIdxShift, (uint32_t)kTabLive)] : 0u;
        if (t == 0) nbs[par * 8 + h] = nbv;
      }
      const bool key0 = SINK && blk == 0 && t == 0 && Lb > 1;
      if (key0) {                                        // key 0's weight stays out of the P operand
#pragma unroll
        for (int hh = 0; hh < GH; ++hh) eh0s[par * 8 + h0 + hh] = (int)e[hh];
      }
      // P^T[head][key] in 8-head x 16-key core matrices: (key / 16) * 256 + (h / 8) * 128 + (h % 8) * 16 + key % 16
      if (!warp_poll(&bars[kDPEmpty + par], ((jj >> 1) & 1) ^ 1, abort_flag, p.err)) bad = true;
      uint8_t* pd = smem + L::kP + par * 2048 + (t >> 4) * 256 + (t & 15);
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {                  // rows >= gq of P^T only feed ignored columns of A
        const int h = h0 + hh;
        if (h < gq) pd[(h >> 3) * 128 + (h & 7) * 16] = (uint8_t)(key0 ? 0u : e[hh]);
      }
#pragma unroll
      for (int hh = 0; hh < GH; ++hh) {
        if (h0 + hh < gq) {
          const uint32_t sum = redux_add_u32(e[hh]);
          if (lane == 0) atomicAdd(&lbsum[par * 8 + h0 + hh], sum);
        }
      }
      fence_async_smem();
      mbar_arrive(&bars[kDPFull + par]);
      if (have_prev && !readout_A(jj - 1, prev_bg, prev_blk)) bad = true;
      have_prev = true;
      prev_bg = bg;
      prev_blk = blk;
      prev_L = Lb;
      ++jj;
    }
    // the last block: its l_b atomics meet at one more barrier, then its partials
    if (have_prev && !bar_any(bar_id, 128, bad || *abort_flag != 0)) {
      write_M(jj - 1, prev_bg, prev_blk, prev_L);
      readout_A(jj - 1, prev_bg, prev_blk);
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDecTmemCols) : "memory");
  }
}

// The committed-order refold of the block partials (reference/lssab8_golden.py:257-335, 350-394):
// one CTA of 64 threads per (head, kv head, sequence), the sequences in the plan's longest-first
// order, so the longest refolds start first and the shortest fill the tail of the grid.  Per
// 32-block segment the partial rows are staged in shared memory with cp.async in one round trip
// while lane u of warp 0 computes block u's fold schedule (the running maximum by a prefix-max
// scan, the rescale distance before the block, its skip distance and term scale) from the
// segment's (NB_b, l_b, e_v) -- prefetched into registers during the previous segment's fold --
// and then thread t folds channels 2t and 2t + 1 with it, one exact multiply-add per block and
// channel, while thread 32 also folds l, in the same order.  A block past the skip window gets
// scale +0, which leaves O bit-identical (O is never -0).
constexpr int kMergeThreads = 64;
template <bool SINK, typename OutT>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(const DecodeArgs p) {
  constexpr int DH = 128;
  __shared__ __align__(16) int sA[kSEG][DH];
  __shared__ int2 sM[kSEG];
  __shared__ int sD[kSEG];                 // rescale distance before block u (0: none)
  __shared__ int sS[kSEG];                 // skip distance of block u
  __shared__ float sSc[kSEG];              // 2^-(s_u + e_v,u), or +0 past the skip window
  __shared__ int sSeg[2];                  // segment -> row: D2, s2
  __shared__ float sLrow;
  pdl_wait();                                          // every block partial is written
  const int h = blockIdx.x, g = blockIdx.y;
  const int b = p.order[blockIdx.z];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int c0 = 2 * t;                                // this thread's channels c0, c0 + 1
  const int gq = p.group;
  const int L = p.seq_lens[b];
  const int nblk = (L + kKB - 1) / kKB;
  if (L <= 0 || nblk > p.max_blocks || (L + 15) / 16 > p.max_pages) return;   // flagged by the plan
  const long long bg = (long long)b * p.KVH + g;
  const int4* pm = p.partM + (bg * p.max_blocks) * gq + h;      // block u's {NB, l_b, eh0} at pm[u * gq]
  const int32_t* evb = p.ev + bg * p.max_blocks;
  int v0a = 0, v0b = 0, evs0 = 0, eh0 = 0;
  if (SINK && L > 1) {
    const int pg = p.block_table[(long long)b * p.max_pages];
    const int8_t* v0 = p.v8p + ((long long)pg * p.KVH + g) * (16 * DH);
    v0a = (int)v0[c0 * 16];
    v0b = (int)v0[(c0 + 1) * 16];
    evs0 = p.ev0[bg];
    eh0 = __ldcg(&pm[0]).z;
  }
  float Oa = 0.0f, Ob = 0.0f, lrow = 0.0f;             // lrow: thread 32 only
  int nbrow = 0;                                       // thread 0 only
  int2 mn = make_int2(INT32_MIN, 0);                   // warp 0: the segment's schedule inputs, one block per lane
  int evn = 0;
  if (w == 0 && lane < min(kSEG, nblk)) {
    mn = __ldcg(reinterpret_cast<const int2*>(&pm[lane * gq]));
    evn = evb[lane];
  }
  for (int s0 = 0; s0 < nblk; s0 += kSEG) {
    const int n = min(kSEG, nblk - s0);
    for (int i = t; i < n * (DH / 4); i += kMergeThreads) {     // 16-byte pieces of the n partial rows
      const int u = i / (DH / 4), q = i % (DH / 4);
      const int32_t* src = p.partA + ((bg * p.max_blocks + s0 + u) * gq + h) * DH + q * 4;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&sA[u][q * 4])), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (w == 0) {
      // ---- the segment's schedule: lane u owns block u
      const bool live = lane < n;
      const int2 m = mn;
      const int ev = evn;
      const int s1 = s0 + kSEG;                              // the next segment's inputs, in flight during the fold
      if (s1 < nblk && lane < min(kSEG, nblk - s1)) {
        mn = __ldcg(reinterpret_cast<const int2*>(&pm[(s1 + lane) * gq]));
        evn = evb[s1 + lane];
      }
      int run = m.x;                                         // inclusive prefix max of NB_b
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run = max(run, y);
      }
      int prev = __shfl_up_sync(0xffffffffu, run, 1);        // running max before block u
      const int nb0 = __shfl_sync(0xffffffffu, m.x, 0);
      if (lane == 0) prev = nb0;                             // block 0 opens the segment
      const int D = live ? m.x - prev : 0;
      const int sg = D > 0 ? 0 : -D;
      const bool add = sg <= kSWIN;
      if (live) {
        sM[lane] = m;
        sD[lane] = D > 0 ? D : 0;
        sS[lane] = sg;
        sSc[lane] = add ? pow2f(-(sg + ev)) : 0.0f;
      }
      // segment -> row (reference/lssab8_golden.py:317-331): the segment's NB is its running max
      const int nbrun = __shfl_sync(0xffffffffu, run, n - 1);
      if (lane == 0) {
        if (s0 == 0) nbrow = nbrun;
        const int D2 = nbrun - nbrow;
        if (D2 > 0) nbrow = nbrun;
        sSeg[0] = D2 > 0 ? D2 : 0;
        sSeg[1] = D2 > 0 ? 0 : -D2;
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int D2 = sSeg[0], s2 = sSeg[1];
    float xa = 0.0f, xb = 0.0f;
    for (int u = 0; u < n; ++u) {
      const int Du = sD[u];
      if (Du > 0) { xa = rescale(xa, Du); xb = rescale(xb, Du); }   // block-uniform branch
      if (SINK && s0 + u == 0 && L > 1) {
        const float sc0 = pow2f(-evs0);
        xa = fold_term(xa, eh0 * v0a, sc0);
        xb = fold_term(xb, eh0 * v0b, sc0);
      }
      const int2 av = *reinterpret_cast<const int2*>(&sA[u][c0]);
      const float sc = sSc[u];
      xa = fold_term(xa, av.x, sc);
      xb = fold_term(xb, av.y, sc);
    }
    if (D2 > 0) { Oa = rescale(Oa, D2); Ob = rescale(Ob, D2); }
    if (s2 <= kSWIN) { Oa = __fadd_rn(Oa, rescale(xa, s2)); Ob = __fadd_rn(Ob, rescale(xb, s2)); }
    if (t == 32) {                                           // l: the same rules, in the same order
      float lseg = 0.0f;
      for (int u = 0; u < n; ++u) {
        const int Du = sD[u];
        if (Du > 0) lseg = rescale(lseg, Du);
        if (sS[u] <= kSWIN) lseg = fold_term(lseg, sM[u].y, pow2f(-sS[u]));
      }
      if (D2 > 0) lrow = rescale(lrow, D2);
      if (s2 <= kSWIN) lrow = __fadd_rn(lrow, rescale(lseg, s2));
      sLrow = lrow;
    }
    __syncthreads();                                         // the stage and schedule are refilled next
  }
  const float lr = sLrow;
  OutT* dst = reinterpret_cast<OutT*>(p.out) + b * p.os0 + (long long)(g * gq + h) * p.os1 + c0 * p.os2;
  dst[0] = from_f32<OutT>(lr != 0.0f ? __fdiv_rn(Oa, lr) : 0.0f);
  dst[p.os2] = from_f32<OutT>(lr != 0.0f ? __fdiv_rn(Ob, lr) : 0.0f);
}

}  // namespace lssab8
