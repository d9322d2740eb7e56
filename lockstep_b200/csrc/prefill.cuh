// LSSA-B8 causal / GQA prefill on sm_100a: tcgen05 int8 MMA with TMEM accumulators.
//
// One CTA = one (batch, query head, 128-row query tile).  It walks the key blocks
// 0 .. tile ASCENDING (the contract's committed order; a descending walk is a different
// function, docs/contract/BLOCK_EXPONENT_VARIANT.md B8.6) with warp-specialised roles:
//
//   warp 0      TMA producer: Q tile once, then K/V 128-key blocks into a 2-stage ring
//               (plain cp.async.bulk.tensor, no multicast).
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_b  = Q8 . K8_b^T   tcgen05.mma kind::i8, s8 x s8 -> s32, M=128 N=128 K=dh
//                 A_b  = P_b . V8_b    tcgen05.mma kind::i8, u8 x s8 -> s32, M=128 N=dh K=128
//               S and A are double-buffered in TMEM (4 x 128 columns = all 512).
//   warps 2-5   "chain" warps, one query row per thread (TMEM lane = row): block max of S,
//               G, NB, the 32-bit chain d = NB - max(S, m - dm) * G (mod 2^32), the T2 gather
//               from an 8 KB zero-padded shared table, l_b = sum eh, and the u8 P row written
//               to shared memory in the SW128 K-major layout the PV MMA reads.
//   warps 6-13  "fold" warps, two threads per row (each owns dh/2 channels): the
//               committed-order binary32 fold of (NB_b, l_b, A_b) into O (registers), the
//               segment -> row fold at 32-block boundaries (O_row in shared memory when a row
//               spans > 1 segment), and the epilogue fl(O / l) -> output dtype.  Both threads
//               of a row run the same scalar recurrence on (NB, l) and disjoint channels.
//
// Exactness: S and A_b are exact integer sums (any MMA order); everything after them is the
// contract's integer chain and a fixed sequence of RN binary32 operations per row
// (reference/lssab8_torch.py:203-271, reference/lssab8_golden.py:257-335).  B9.1 sink_alone
// (reference/lssab9_torch.py:276-304): key 0's weight is removed from block 0's P operand
// (l_b keeps it) and its product eh0 * v8[0] is folded first with e_v0.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace lssab8 {

struct PrefillArgs {
  int B, H, KVH, T, dh, Tpad, nblk, group;
  const int32_t* eq;    // [B, H, Tpad]
  const int32_t* ek;    // [B, KVH, nblk]
  const int32_t* ev;    // [B, KVH, nblk]
  const int32_t* ev0;   // [B, KVH] (sink) or nullptr
  const int8_t* v8;     // [B, KVH, Tpad, dh] (sink: key 0's row)
  void* out;            // output, element strides below
  long long os0, os1, os2, os3;   // out[b, t, h, c]
  int out_dtype;
  uint32_t gbase;
  int* err;
};

// -------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor (sm_100 layout: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
// version 1 at bit 46, swizzle mode [61,64): 2 = 128B, 4 = 64B).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swz) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)swz << 61);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A/B format 1 = s8, 0 = u8
// (bits 7-9, 10-12), A/B major 0 = K, 1 = MN (bits 15, 16), N>>3 (bits 17-22), M>>4 (24-28).
__host__ __device__ constexpr uint32_t idesc_i8(int a_signed, int b_signed, int b_mn_major, int M, int N) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------ smem layout
template <int DH>
struct PrefillSmem {
  static constexpr int kTile = 128 * DH;                 // one Q/K/V tile, bytes
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;                       // 2 stages
  static constexpr int kV = 3 * kTile;                   // 2 stages
  static constexpr int kP = 5 * kTile;                   // 2 x 16 KB, SW128 K-major u8
  static constexpr int kTab = kP + 2 * 16384;            // 8 KB zero-padded T2
  static constexpr int kInfo = kTab + kTabPad;           // 2 x 128 x int4
  static constexpr int kV0 = kInfo + 2 * 128 * 16;       // key 0's int8 value row (sink)
  static constexpr int kBar = kV0 + 256;                 // mbarriers
  static constexpr int kNumBars = 25;
  static constexpr int kMisc = kBar + 256;               // tmem base, abort flag
  static constexpr int kORow = kMisc + 64;               // [DH][128] f32 (multi-segment rows)
  static constexpr int kBytesSingle = kORow;
  static constexpr int kBytesMulti = kORow + DH * 128 * 4;
};

__device__ const uint8_t kT2Live[kTabLive] = {
#include "t2_table.inc"
};

enum BarId : int {
  kBarQ = 0, kBarKFull = 1, kBarKEmpty = 3, kBarVFull = 5, kBarVEmpty = 7, kBarSFull = 9, kBarSEmpty = 11,
  kBarPFull = 13, kBarPEmpty = 15, kBarAFull = 17, kBarAEmpty = 19, kBarIFull = 21, kBarIEmpty = 23
};

template <int DH, bool SINK, typename OutT, bool MULTI>
__global__ void __launch_bounds__(448, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const PrefillArgs p) {
  constexpr bool multi_seg = MULTI;    // rows spanning more than one 32-block segment
  using L = PrefillSmem<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // 1024-B aligned, still __shared__
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);
  uint8_t* tab = smem + L::kTab;
  int4* info = reinterpret_cast<int4*>(smem + L::kInfo);
  int8_t* v0row = reinterpret_cast<int8_t*>(smem + L::kV0);
  float* orow = reinterpret_cast<float*>(smem + L::kORow);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile = gridDim.x;
  const int tile = ntile - 1 - (int)blockIdx.x;      // longest rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / p.group;
  const int nb = tile + 1;                           // causal: blocks 0 .. tile
  const int qrow0 = (b * p.H + h) * p.Tpad + tile * 128;
  const int krow0 = (b * p.KVH + g) * p.Tpad;

  // ---- setup: table, barriers, TMEM
  for (int i = threadIdx.x; i < kTabPad; i += blockDim.x) tab[i] = (i < kTabLive) ? kT2Live[i] : 0;
  if (SINK && threadIdx.x < DH) v0row[threadIdx.x] = p.v8[(long long)krow0 * DH + threadIdx.x];
  if (threadIdx.x == 0) {
    mbar_init(&bars[kBarQ], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kBarKFull + s], 1);  mbar_init(&bars[kBarKEmpty + s], 1);
      mbar_init(&bars[kBarVFull + s], 1);  mbar_init(&bars[kBarVEmpty + s], 1);
      mbar_init(&bars[kBarSFull + s], 1);  mbar_init(&bars[kBarSEmpty + s], 128);
      mbar_init(&bars[kBarPFull + s], 128); mbar_init(&bars[kBarPEmpty + s], 1);
      mbar_init(&bars[kBarAFull + s], 1);  mbar_init(&bars[kBarAEmpty + s], 256);
      mbar_init(&bars[kBarIFull + s], 128); mbar_init(&bars[kBarIEmpty + s], 256);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if constexpr (MULTI) {
    for (int i = threadIdx.x; i < DH * 128; i += blockDim.x) orow[i] = 0.0f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bars[kBarQ], L::kTile);
      tma_load_2d(smem + L::kQ, &tm_q, 0, qrow0, &bars[kBarQ]);
      for (int j = 0; j < nb; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bars[kBarKEmpty + s], ph ^ 1, abort_flag, p.err)) break;
        mbar_expect_tx(&bars[kBarKFull + s], L::kTile);
        tma_load_2d(smem + L::kK + s * L::kTile, &tm_k, 0, krow0 + j * 128, &bars[kBarKFull + s]);
        if (!mbar_wait(&bars[kBarVEmpty + s], ph ^ 1, abort_flag, p.err)) break;
        mbar_expect_tx(&bars[kBarVFull + s], L::kTile);
        tma_load_2d(smem + L::kV + s * L::kTile, &tm_v, 0, krow0 + j * 128, &bars[kBarVFull + s]);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kSwz = (DH == 128) ? 2u : 4u;          // 128B / 64B swizzle
      constexpr uint32_t kRowGroup = 8 * DH;                    // bytes per 8 rows of a tile
      constexpr uint32_t idesc_qk = idesc_i8(1, 1, 0, 128, 128);
      constexpr uint32_t idesc_pv = idesc_i8(0, 1, 1, 128, DH);
      const uint32_t sq = smem_u32(smem + L::kQ);
      bool ok = mbar_wait(&bars[kBarQ], 0, abort_flag, p.err);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bars[kBarKFull + s], ph, abort_flag, p.err)) return false;
        if (!mbar_wait(&bars[kBarSEmpty + s], ph ^ 1, abort_flag, p.err)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + L::kK + s * L::kTile);
#pragma unroll
        for (int kk = 0; kk < DH / 32; ++kk) {
          umma_i8(tmem + s * 128, umma_desc(sq + kk * 32, 16, kRowGroup, kSwz),
                  umma_desc(sk + kk * 32, 16, kRowGroup, kSwz), idesc_qk, kk > 0);
        }
        umma_commit(&bars[kBarSFull + s]);
        umma_commit(&bars[kBarKEmpty + s]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < nb; ++j) {
        if (j + 1 < nb && !issue_qk(j + 1)) break;
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bars[kBarPFull + s], ph, abort_flag, p.err)) break;
        if (!mbar_wait(&bars[kBarVFull + s], ph, abort_flag, p.err)) break;
        if (!mbar_wait(&bars[kBarAEmpty + s], ph ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + L::kP + s * 16384);
        const uint32_t sv = smem_u32(smem + L::kV + s * L::kTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // A = P (K-major SW128, 32 keys = 32 bytes per step); B = V (MN-major: 32 keys =
          // 4 groups of 8 rows per step; LBO = MN-atom stride (one atom), SBO = 8-row stride)
          umma_i8(tmem + 256 + s * 128, umma_desc(sp + kk * 32, 16, 1024, 2),
                  umma_desc(sv + kk * 32 * DH, L::kTile, kRowGroup, kSwz), idesc_pv, kk > 0);
        }
        umma_commit(&bars[kBarAFull + s]);
        umma_commit(&bars[kBarVEmpty + s]);
        umma_commit(&bars[kBarPEmpty + s]);
      }
    }
  } else if (warp < 6) {
    // ================================================================ chain warps
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lanebase = (uint32_t)(q4 * 32) << 16;
    const int eqr = p.eq[(long long)qrow0 + r];
    const int32_t* ekg = p.ek + (long long)(b * p.KVH + g) * p.nblk;
    const uint32_t prow = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    for (int j = 0; j < nb; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait_warp(&bars[kBarSFull + s], ph, abort_flag, p.err)) break;
      tc_fence_after();
      const bool diag = (j == tile);                     // key c of the diagonal block visible iff c <= r
      const uint32_t sbase = tmem + lanebase + s * 128;
      // pass 1: exact block max over the visible keys (32 TMEM columns at a time)
      int m = INT32_MIN;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t v[32];
        tmem_ld32(sbase + cc * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) if (diag && cc * 32 + c > r) v[c] = 0x80000000u;
        int m2 = (int)v[0];
#pragma unroll
        for (int c = 1; c < 31; c += 2) m2 = __vimax3_s32(m2, (int)v[c], (int)v[c + 1]);
        m = __vimax3_s32(m, m2, (int)v[31]);
      }
      const uint32_t G = g_fold(p.gbase, eqr + ekg[j]);
      const int nbv = nb_of(m, G);
      const uint32_t NBlo = (uint32_t)nbv << kBHI;
      const int lg = 31 - __clz((int)G);
      const int dm = 1 << max(0, 30 - lg);              // dm * G in [2^30, 2^31): >= 9 doublings
      const int lo = m - dm;
      const uint32_t negG = 0u - G;
      if (!mbar_wait_warp(&bars[kBarPEmpty + s], ph ^ 1, abort_flag, p.err)) break;
      const uint32_t pbase = smem_u32(smem + L::kP + s * 16384) + prow;
      uint32_t lb = 0, eh0 = 0;
      // pass 2: the chain and the u8 P row (two 16-key chunks per 32 columns)
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t v[32];
        tmem_ld32(sbase + cc * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) if (diag && cc * 32 + c > r) v[c] = 0x80000000u;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t w[4];
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            uint32_t acc = 0;
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              const int sc = max((int)v[half * 16 + qq * 4 + x], lo);
              const uint32_t d = NBlo + (uint32_t)sc * negG;   // exact: d < 2^32
              acc |= (uint32_t)tab[d >> kIdxShift] << (8 * x);
            }
            w[qq] = acc;
            lb = __dp4a(acc, 0x01010101u, lb);
          }
          const int chunk = cc * 2 + half;
          if (SINK && chunk == 0 && j == 0 && p.T > 1) { eh0 = w[0] & 0xFFu; w[0] &= ~0xFFu; }
          st_shared_v4(pbase + (uint32_t)((chunk ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarSEmpty + s]);
      fence_async_smem();
      mbar_arrive(&bars[kBarPFull + s]);
      if (!mbar_wait_warp(&bars[kBarIEmpty + s], ph ^ 1, abort_flag, p.err)) break;
      info[s * 128 + r] = make_int4(nbv, (int)lb, (int)eh0, 0);
      mbar_arrive(&bars[kBarIFull + s]);
    }
  } else {
    // ================================================================ fold warps
    constexpr int HD = DH / 2;                        // channels owned by this thread
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int c0 = (warp >= 10) ? HD : 0;
    const uint32_t lanebase = (uint32_t)(q4 * 32) << 16;
    const int32_t* evg = p.ev + (long long)(b * p.KVH + g) * p.nblk;
    const int ev0 = SINK ? p.ev0[b * p.KVH + g] : 0;
    float O[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) O[c] = 0.0f;
    float lseg = 0.0f, lrow = 0.0f;
    int nbrun = 0, nbrow = 0;
    bool have_seg = false, have_row = false;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait_warp(&bars[kBarIFull + s], ph, abort_flag, p.err)) { ok = false; break; }
      const int4 inf = info[s * 128 + r];
      mbar_arrive(&bars[kBarIEmpty + s]);
      const int nbb = inf.x;
      if (!have_seg) { nbrun = nbb; have_seg = true; }
      const int D = nbb - nbrun;
      int sg = 0;
      if (D > 0) {
#pragma unroll
        for (int c = 0; c < HD; ++c) O[c] = rescale(O[c], D);
        lseg = rescale(lseg, D);
        nbrun = nbb;
      } else {
        sg = -D;
      }
      if (!mbar_wait_warp(&bars[kBarAFull + s], ph, abort_flag, p.err)) { ok = false; break; }
      tc_fence_after();
      if (sg <= kSWIN) {
        if (SINK && j == 0 && p.T > 1) {
          const float sc0 = pow2f(-(sg + ev0));
          const int e0w = inf.z;
#pragma unroll
          for (int c = 0; c < HD; ++c) O[c] = fold_term(O[c], e0w * (int)v0row[c0 + c], sc0);
        }
        const float scO = pow2f(-(sg + evg[j]));
#pragma unroll
        for (int cc = 0; cc < HD / 16; ++cc) {
          uint32_t a[16];
          tmem_ld16(tmem + lanebase + 256 + s * 128 + c0 + cc * 16, a);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c) O[cc * 16 + c] = fold_term(O[cc * 16 + c], (int)a[c], scO);
        }
        lseg = fold_term(lseg, inf.y, pow2f(-sg));
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarAEmpty + s]);
      const bool seg_end = ((j + 1) % kSEG == 0) || (j == nb - 1);
      if (MULTI && seg_end) {
        // segment -> row: the same three rules (reference/lssab8_golden.py:317-331)
        if (!have_row) { nbrow = nbrun; have_row = true; }
        const int D2 = nbrun - nbrow;
        int s2 = 0;
        if (D2 > 0) {
#pragma unroll 8
          for (int c = c0; c < c0 + HD; ++c) orow[c * 128 + r] = rescale(orow[c * 128 + r], D2);
          lrow = rescale(lrow, D2);
          nbrow = nbrun;
        } else {
          s2 = -D2;
        }
        if (s2 <= kSWIN) {
#pragma unroll
          for (int c = 0; c < HD; ++c) orow[(c0 + c) * 128 + r] = __fadd_rn(orow[(c0 + c) * 128 + r], rescale(O[c], s2));
          lrow = __fadd_rn(lrow, rescale(lseg, s2));
        }
#pragma unroll
        for (int c = 0; c < HD; ++c) O[c] = 0.0f;
        lseg = 0.0f;
        have_seg = false;
      }
    }
    // ---- epilogue: out = O_row / l_row (one RN division), l_row == 0 -> 0
    const int i = tile * 128 + r;
    if (ok && i < p.T) {
      if constexpr (!MULTI) {
        // a single segment: O_row = 0 + rescale(O_seg, 0), l_row likewise
#pragma unroll
        for (int c = 0; c < HD; ++c) O[c] = rescale(O[c], 0);
        lrow = rescale(lseg, 0);
      } else {
#pragma unroll
        for (int c = 0; c < HD; ++c) O[c] = orow[(c0 + c) * 128 + r];
      }
      OutT* dst = reinterpret_cast<OutT*>(p.out) + b * p.os0 + (long long)i * p.os1 + h * p.os2 + c0 * p.os3;
      const bool nz = (lrow != 0.0f);
#pragma unroll
      for (int c = 0; c < HD; ++c) dst[c * p.os3] = from_f32<OutT>(nz ? __fdiv_rn(O[c], lrow) : 0.0f);
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace lssab8
