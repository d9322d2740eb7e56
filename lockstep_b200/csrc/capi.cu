// C ABI of liblssab8_b200.so (declarations and contracts: include/lssab8.h).
//
// Host-side responsibilities: argument validation (every error is a status code, never an
// exception), TMA tensor-map encoding, workspace carving, kernel instantiation by
// (head dim, sink, output dtype), and the per-device error word.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <utility>
#include <cstring>
#include <mutex>

#include "../../include/lssab8.h"
#include "common.cuh"
#include "prep.cuh"
#include "prefill.cuh"
#include "decode.cuh"
#include "decode_tc.cuh"

using namespace lssab8;

namespace {

constexpr const char* kVersion = "0.1.0";

// ------------------------------------------------------------------ device error word
__device__ int g_dev_err;

struct DevState {
  int* err = nullptr;
  bool prefill_attr_set = false;
  int num_sms = 0;
};
std::mutex g_mu;
DevState g_dev[64];

int dev_state(DevState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrCuda;
  std::lock_guard<std::mutex> lk(g_mu);
  DevState& st = g_dev[dev];
  if (!st.err) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) return kErrCuda;
    st.err = static_cast<int*>(p);
  }
  if (st.num_sms <= 0 && cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kErrCuda;
  *out = &st;
  return kOk;
}

// ------------------------------------------------------------------ TMA encode (driver API)
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encode() {
  static std::once_flag once;
  static int rc = kOk;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      rc = kErrCuda;
      return;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return rc;
}

// rows x dh int8 matrix, box 128 rows x dh, swizzle = dh bytes
// 2-D int8 tensor map over [rows, dh] (row pitch dh bytes), boxes of box_rows x dh, swizzled for
// the UMMA K-major layouts (128B swizzle at dh 128, 64B at dh 64).
int make_tmap(CUtensorMap* tm, const void* base, long long rows, int dh, int box_rows = 128) {
  if (get_encode() != kOk) return kErrCuda;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return kErrArg;
  cuuint64_t dims[2] = {(cuuint64_t)dh, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)dh};
  cuuint32_t box[2] = {(cuuint32_t)dh, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        dh == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrCuda;
}

inline int cuda_rc(cudaError_t e) { return e == cudaSuccess ? kOk : kErrCuda; }
inline int launch_rc() { return cuda_rc(cudaGetLastError()); }

uint32_t gbase_of(int dh) {
  // round(2^26 / (sqrt(dh) ln 2)) with round-half-even, as Python's round() on the double
  // (reference/lssab_golden.py:161).
  double x = std::ldexp(1.0, kBHI) / (std::sqrt((double)dh) * std::log(2.0));
  return (uint32_t)std::nearbyint(x);
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline int tpad_of(int T) { return ((T + 127) / 128) * 128; }

// ------------------------------------------------------------------ sha256 (FIPS 180-4)
struct Sha256 {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint8_t buf[64];
  uint64_t len = 0;
  size_t n = 0;
  static uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }
  void block(const uint8_t* p) {
    static const uint32_t K[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98,
        0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786,
        0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8,
        0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13,
        0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819,
        0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a,
        0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
        0xc67178f2};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      uint32_t ch = (e & f) ^ (~e & g);
      uint32_t t1 = hh + S1 + ch + K[i] + w[i];
      uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      uint32_t t2 = S0 + mj;
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const void* data, size_t m) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    len += m;
    while (m--) {
      buf[n++] = *p++;
      if (n == 64) { block(buf); n = 0; }
    }
  }
  void final(char* hex) {
    uint64_t bits = len * 8;
    uint8_t pad = 0x80;
    update(&pad, 1);
    uint8_t z = 0;
    while (n != 56) update(&z, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = (uint8_t)(bits >> (56 - 8 * i));
    for (int i = 0; i < 8; ++i) { buf[n++] = lb[i]; }
    block(buf);
    for (int i = 0; i < 8; ++i) std::snprintf(hex + 8 * i, 9, "%08x", h[i]);
  }
};

const uint8_t kT2Host[kTabLive] = {
#include "t2_table.inc"
};

// ------------------------------------------------------------------ kernel dispatch helpers
template <typename F>
int with_in_dtype(int dtype, F&& f) {
  switch (dtype) {
    case kF32: return f((const float*)nullptr);
    case kF16: return f((const __half*)nullptr);
    case kBF16: return f((const __nv_bfloat16*)nullptr);
    default: return kErrArg;
  }
}

// Launch with programmatic dependent launch: the kernel may start while the previous kernel on
// the stream finishes; it executes griddepcontrol.wait before it reads that kernel's output.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kfn)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_rc(cudaLaunchKernelEx(&cfg, kfn, std::forward<Args>(args)...));
}

template <int DH, bool SINK, typename OutT, bool GEN = false, bool KS = false>
int launch_prefill_t(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PrefillArgs& a,
                     int num_sms, cudaStream_t st) {
  using L = PrefillSmem<DH>;
  const int multi = a.nblk > kSEG;                         // rows span more than one fold segment
  // the T2 copies, the aligned tiles; at least ~116 KB so only one CTA (and one 512-column TMEM
  // allocation) lands on an SM
  int smem = kTabBytes + 1024 + L::kBytes;
  if (smem < 116 * 1024) smem = 116 * 1024;
  auto kfn = multi ? prefill_kernel<DH, SINK, OutT, true, GEN, KS> : prefill_kernel<DH, SINK, OutT, false, GEN, KS>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return kErrCuda;
  const long long items = (long long)(a.Tpad / 128) * a.H * a.B;      // persistent: one CTA per SM
  const int grid = (int)std::min<long long>(items, (long long)std::max(num_sms, 1));
  return launch_pdl(kfn, dim3(grid), dim3(kPrefillThreads), smem, st, tq, tk, tv, a);
}

template <int DH, bool SINK>
int launch_prefill_out(int out_dtype, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                       const PrefillArgs& a, int num_sms, cudaStream_t st) {
  switch (out_dtype) {
    case kF32: return launch_prefill_t<DH, SINK, float>(tq, tk, tv, a, num_sms, st);
    case kF16: return launch_prefill_t<DH, SINK, __half>(tq, tk, tv, a, num_sms, st);
    case kBF16: return launch_prefill_t<DH, SINK, __nv_bfloat16>(tq, tk, tv, a, num_sms, st);
    default: return kErrArg;
  }
}

template <int DH, bool SINK, typename OutT>
int launch_decode_t(const DecodeArgs& a, int max_splits, cudaStream_t st) {
  using L = DecodeSmem<DH>;
  const int smem = L::kBytes + 128;
  auto kfn = decode_kernel<DH, SINK, OutT>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return kErrCuda;
  dim3 grid(max_splits, a.KVH, a.B);
  kfn<<<grid, 128, smem, st>>>(a);
  return launch_rc();
}

template <int DH, bool SINK>
int launch_decode_out(int out_dtype, const DecodeArgs& a, int max_splits, cudaStream_t st) {
  switch (out_dtype) {
    case kF32: return launch_decode_t<DH, SINK, float>(a, max_splits, st);
    case kF16: return launch_decode_t<DH, SINK, __half>(a, max_splits, st);
    case kBF16: return launch_decode_t<DH, SINK, __nv_bfloat16>(a, max_splits, st);
    default: return kErrArg;
  }
}

template <bool SINK, typename OutT, int GQ>
int launch_decode_tc_t(const DecodeArgs& a, int max_splits, int num_sms, cudaStream_t st) {
  CUtensorMap tk, tq;
  int rc;
  if ((rc = make_tmap(&tk, a.k8p, (long long)a.num_pages * a.KVH * 16, 128, 16))) return rc;
  if ((rc = make_tmap(&tq, a.q8, (long long)a.B * a.H, 128, 16))) return rc;
  const int smem = DecTcSmem::kBytes + 1024;
  auto kfn = decode_tc_kernel<SINK, OutT, GQ>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return kErrCuda;
  (void)max_splits;     // exact block partials: the streaming kernel schedules blocks, not splits
  // the live block count is known on the device only; the grid covers the most there can be
  const long long chunks = ((long long)a.B * a.KVH * a.max_blocks + kDecChunk - 1) / kDecChunk;
  const int grid = (int)std::min<long long>(chunks, 2LL * std::max(num_sms, 1));   // two CTAs per SM
  if ((rc = launch_pdl(kfn, dim3(grid), dim3(DecWorkers<GQ>::kThreads), smem, st, tk, tq, a))) return rc;
  // heads fastest, then kv heads, then the sequences in the plan's longest-first order
  return launch_pdl(decode_merge_kernel<SINK, OutT>, dim3(a.group, a.KVH, a.B), dim3(kMergeThreads), 0, st, a);
}

template <bool SINK>
int launch_decode_tc_out(int out_dtype, const DecodeArgs& a, int max_splits, int num_sms, cudaStream_t st) {
  switch (out_dtype) {
    case kF32: return a.group == 4 ? launch_decode_tc_t<SINK, float, 4>(a, max_splits, num_sms, st)
                                   : launch_decode_tc_t<SINK, float, 8>(a, max_splits, num_sms, st);
    case kF16: return a.group == 4 ? launch_decode_tc_t<SINK, __half, 4>(a, max_splits, num_sms, st)
                                   : launch_decode_tc_t<SINK, __half, 8>(a, max_splits, num_sms, st);
    case kBF16: return a.group == 4 ? launch_decode_tc_t<SINK, __nv_bfloat16, 4>(a, max_splits, num_sms, st)
                                    : launch_decode_tc_t<SINK, __nv_bfloat16, 8>(a, max_splits, num_sms, st);
    default: return kErrArg;
  }
}

// the vectorised quantisers need a contiguous channel dim, dh in {64, 128} and 16-byte aligned
// rows (base and every stride a multiple of 16 bytes)
template <typename InT>
bool vec_ok(const void* x, const Strides4& s, int dh) {
  const long long e = (long long)sizeof(InT);
  return (dh == 64 || dh == 128) && s.s3 == 1 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
         (s.s0 * e) % 16 == 0 && (s.s1 * e) % 16 == 0 && (s.s2 * e) % 16 == 0;
}

bool strides_ok(const int64_t* s, int n) {
  if (!s) return false;
  for (int i = 0; i < n; ++i) if (s[i] < 0) return false;
  return true;
}

struct PrefillWs {
  size_t q8, eq, k8, ek, v8, ev, ev0, total;
};

PrefillWs prefill_ws(int B, int H, int KVH, int T, int dh) {
  PrefillWs w{};
  const size_t Tpad = (size_t)tpad_of(T), nblk = Tpad / 128;
  size_t o = 0;
  w.q8 = o; o += align256((size_t)B * H * Tpad * dh);
  w.eq = o; o += align256((size_t)B * H * Tpad * 4);
  w.k8 = o; o += align256((size_t)B * KVH * Tpad * dh);
  w.ek = o; o += align256((size_t)B * KVH * nblk * 4);
  w.v8 = o; o += align256((size_t)B * KVH * Tpad * dh);
  w.ev = o; o += align256((size_t)B * KVH * nblk * 4);
  w.ev0 = o; o += align256((size_t)B * KVH * 4);
  w.total = o + 256;     // slack for aligning the caller's base
  return w;
}

struct DecodeWs {
  size_t q8, eq, partA, partM, tickets, blk_off, order, total;
};

DecodeWs decode_ws(int B, int H, int KVH, int dh, int max_blocks) {
  DecodeWs w{};
  const int gq = H / KVH;
  size_t o = 0;
  w.q8 = o; o += align256((size_t)B * H * dh);
  w.eq = o; o += align256((size_t)B * H * 4);
  w.partA = o; o += align256((size_t)B * KVH * max_blocks * gq * dh * 4);
  w.partM = o; o += align256((size_t)B * KVH * max_blocks * gq * 16);
  w.tickets = o; o += align256((size_t)B * KVH * 4);
  w.blk_off = o; o += align256((size_t)(B + 1) * 4);         // the live-block plan
  w.order = o; o += align256((size_t)B * 4);                 // the refold's sequence order
  w.total = o + 256;
  return w;
}

bool shape_ok(int B, int H, int KVH, int T, int dh) {
  return B > 0 && H > 0 && KVH > 0 && T > 0 && dh > 0 && H % KVH == 0 && dh <= 256 && dh % 32 == 0 &&
         (long long)T <= (1ll << 24);
}

}  // namespace

// the prefill epilogue's division (div_chunk with the row reciprocal) of y[i] by l[i], one element
// per thread: the pair (y[i], y[i]) takes the paired path when y[i] and l[i] lie in the Markstein
// window and the scalar one otherwise
__global__ void selftest_div_kernel(const float* y, const float* l, long long n, float* out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float li = l[i];
    float q[4] = {y[i], y[i], y[i], y[i]};
    div_chunk<4, false>(q, li, __frcp_rn(li), div_window(li));
    out[i] = q[0];
  }
}

// the prefill fold's rescale (rescale_channels) of the pair x[2i], x[2i + 1] by D[i], then the
// fold's fused multiply-add of a zero term with a positive scale, one pair per thread
__global__ void selftest_rescale_kernel(const float* x, const int* D, long long npairs, float* out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npairs; i += (long long)gridDim.x * blockDim.x) {
    const int d = D[i];
    const float sc = pow2f(-min(max(d, 0), 126));
    uint32_t o[2] = {__float_as_uint(x[2 * i]), __float_as_uint(x[2 * i + 1])};
    rescale_channels<2>(o, d, f2_pack(sc, sc));
    float lo, hi;
    f2_unpack(f2_fma(f2_pack(0.0f, 0.0f), f2_pack(1.0f, 1.0f), f2_pack(__uint_as_float(o[0]), __uint_as_float(o[1]))), lo, hi);
    out[2 * i] = lo;
    out[2 * i + 1] = hi;
  }
}

// Causal prefill of query rows [T0, T) (T0 a multiple of 128) against the key lattice of [0, T):
// q8/eq hold the chunk's rows (Tpad = tpad(T - T0)), k8/v8/ek/ev the whole prefix
// (Tpad = tpad(T)), out the chunk's T - T0 rows.  T0 = 0 is the whole prefill.
static int prefill_lattice_impl(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek, const int8_t* v8,
                         const int32_t* ev, const int32_t* ev0, int B, int H, int KVH, int T0, int T, int dh,
                         float* orow_scratch, void* out, int out_dtype, const int64_t* os, void* stream,
                         uint64_t wait_ns = kWaitLimitNs, int withhold = -1, int npeers = 0,
                         void* const* peers = nullptr, int general = 0, int causal = 1,
                         const uint32_t* kmask = nullptr, const int8_t* d8 = nullptr) {
  if (!q8 || !eq || !k8 || !ek || !v8 || !ev || !out || !shape_ok(B, H, KVH, T, dh) || !strides_ok(os, 4))
    return kErrArg;
  if (dh != 64 && dh != 128) return kErrUnsupported;
  const int TpadQ = tpad_of(T - T0), TpadK = tpad_of(T);
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_tmap(&tq, q8, (long long)B * H * TpadQ, dh))) return rc;
  if ((rc = make_tmap(&tk, k8, (long long)B * KVH * TpadK, dh))) return rc;
  if ((rc = make_tmap(&tv, v8, (long long)B * KVH * TpadK, dh))) return rc;
  PrefillArgs a{};
  a.B = B; a.H = H; a.KVH = KVH; a.T = T; a.dh = dh; a.Tpad = TpadQ; a.nblk = TpadK / 128; a.group = H / KVH;
  a.tile0 = T0 / 128;
  a.eq = eq; a.ek = ek; a.ev = ev; a.ev0 = ev0; a.v8 = v8;
  a.out = out; a.os0 = os[0]; a.os1 = os[1]; a.os2 = os[2]; a.os3 = os[3]; a.out_dtype = out_dtype;
  a.orow = orow_scratch;
  a.gbase = gbase_of(dh);
  a.mul_entry = kTabCopies * 4;
  a.mul_b1 = 1u << 8;
  a.mul_b2 = 1u << 16;
  a.mul_b3 = 1u << 24;
  a.err = ds->err;
  a.wait_ns = wait_ns;
  a.withhold = withhold;
  if (npeers < 0 || npeers > kMaxPeers || (npeers > 0 && !peers)) return kErrArg;
  a.npeers = npeers;
  for (int i = 0; i < npeers; ++i) {
    // same alignment as out modulo 16 bytes, so the vectorised stores apply to every copy
    if (!peers[i] || ((reinterpret_cast<uintptr_t>(peers[i]) ^ reinterpret_cast<uintptr_t>(out)) & 15)) return kErrArg;
    a.peers[i] = peers[i];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool sink = ev0 != nullptr;
  if (d8) {                                          // B9.3: the shifted PV weights (bf16 / f32 out)
    if (general || npeers || (out_dtype != kF32 && out_dtype != kBF16)) return kErrArg;
    a.causal = 1;
    a.d8 = d8;
    if (out_dtype == kF32) {
      if (dh == 128) return sink ? launch_prefill_t<128, true, float, false, true>(tq, tk, tv, a, ds->num_sms, st)
                                 : launch_prefill_t<128, false, float, false, true>(tq, tk, tv, a, ds->num_sms, st);
      return sink ? launch_prefill_t<64, true, float, false, true>(tq, tk, tv, a, ds->num_sms, st)
                  : launch_prefill_t<64, false, float, false, true>(tq, tk, tv, a, ds->num_sms, st);
    }
    if (dh == 128)
      return sink ? launch_prefill_t<128, true, __nv_bfloat16, false, true>(tq, tk, tv, a, ds->num_sms, st)
                  : launch_prefill_t<128, false, __nv_bfloat16, false, true>(tq, tk, tv, a, ds->num_sms, st);
    return sink ? launch_prefill_t<64, true, __nv_bfloat16, false, true>(tq, tk, tv, a, ds->num_sms, st)
                : launch_prefill_t<64, false, __nv_bfloat16, false, true>(tq, tk, tv, a, ds->num_sms, st);
  }
  if (general) {                                     // float32 out; causal flag and key mask
    if (out_dtype != kF32 || !kmask || T0 != 0 || npeers) return kErrArg;
    a.causal = causal ? 1 : 0;
    a.kmask = kmask;
    if (dh == 128) return sink ? launch_prefill_t<128, true, float, true>(tq, tk, tv, a, ds->num_sms, st)
                               : launch_prefill_t<128, false, float, true>(tq, tk, tv, a, ds->num_sms, st);
    return sink ? launch_prefill_t<64, true, float, true>(tq, tk, tv, a, ds->num_sms, st)
                : launch_prefill_t<64, false, float, true>(tq, tk, tv, a, ds->num_sms, st);
  }
  a.causal = 1;
  if (dh == 128) return sink ? launch_prefill_out<128, true>(out_dtype, tq, tk, tv, a, ds->num_sms, st)
                             : launch_prefill_out<128, false>(out_dtype, tq, tk, tv, a, ds->num_sms, st);
  return sink ? launch_prefill_out<64, true>(out_dtype, tq, tk, tv, a, ds->num_sms, st)
              : launch_prefill_out<64, false>(out_dtype, tq, tk, tv, a, ds->num_sms, st);
}

// ========================================================================== extern "C"
extern "C" {

int lssab8_version(char* buf, int buflen) {
  if (!buf || buflen < 128) return kErrArg;
  Sha256 s;
  char num[8];
  for (int k = 0; k < 17 * 128; ++k) {
    int v = k < kTabLive ? kT2Host[k] : 0;
    int n = std::snprintf(num, sizeof num, k ? ",%d" : "%d", v);
    s.update(num, (size_t)n);
  }
  char hex[65];
  s.final(hex);
  std::snprintf(buf, (size_t)buflen, "lssab8-b200 %s T2=%s", kVersion, hex);
  return kOk;
}

const char* lssab8_strerror(int code) {
  switch (code) {
    case kOk: return "ok";
    case kErrArg: return "invalid argument (shape, stride, dtype or pointer)";
    case kErrUnsupported: return "unsupported by the B200 kernels (head dim / group size)";
    case kErrCuda: return "CUDA error";
    case kErrWorkspace: return "workspace too small";
    case kErrDevice: return "device error word set";
    case LSSAB8_ESCRATCH: return "problem needs more scratch than the fixed no-alloc buffer";
    default: return "unknown status";
  }
}

int lssab8_device_errors(int clear, void* stream, int* bits) {
  if (!bits) return kErrArg;
  DevState* st = nullptr;
  int rc = dev_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  if (cudaMemcpyAsync(&host, st->err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return kErrCuda;
  if (cudaStreamSynchronize(s) != cudaSuccess) return kErrCuda;
  *bits = host;
  if (clear && host) {
    if (cudaMemsetAsync(st->err, 0, sizeof(int), s) != cudaSuccess) return kErrCuda;
    if (cudaStreamSynchronize(s) != cudaSuccess) return kErrCuda;
  }
  return kOk;
}

// The decode's query quantiser ([B, H, dh] rows): the vector kernel is launched with
// programmatic dependent launch, so it runs beside the decode plan kernel before it (which it does
// not read); it waits for the plan before it completes, so the streaming kernel's wait on it
// covers the plan too.  Other layouts take lssab8_quant_rows.
static int quant_queries_pdl(const void* q, int dtype, int B, int H, int dh, const int64_t* q4, int8_t* q8,
                             int32_t* eq, cudaStream_t st) {
  Strides4 s{q4[0], q4[1], q4[2], q4[3]};
  return with_in_dtype(dtype, [&](auto tag) -> int {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    if (!vec_ok<InT>(q, s, dh)) return lssab8_quant_rows(q, dtype, B, H, 1, dh, q4, 1, q8, eq, st);
    constexpr int N = Vec16<InT>::kN;
    const int rpw = 32 / (dh / N);
    const long long per_cta = 8LL * rpw * kRowsPerLane;
    const int grid = (int)(((long long)B * H + per_cta - 1) / per_cta);
    if (dh == 128)
      return launch_pdl(quant_rows_vec_kernel<InT, 128>, dim3(grid), dim3(256), 0, st, static_cast<const InT*>(q), s, B,
                        H, 1, 1, q8, eq);
    return launch_pdl(quant_rows_vec_kernel<InT, 64>, dim3(grid), dim3(256), 0, st, static_cast<const InT*>(q), s, B, H,
                      1, 1, q8, eq);
  });
}

int lssab8_quant_rows(const void* x, int dtype, int B, int H, int T, int dh, const int64_t* xs, int Tpad,
                      int8_t* q8, int32_t* eq, void* stream) {
  if (!x || !q8 || !eq || !shape_ok(B, H, H, T, dh) || Tpad < T || !strides_ok(xs, 4)) return kErrArg;
  Strides4 s{xs[0], xs[1], xs[2], xs[3]};
  const long long rows = (long long)B * H * Tpad;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    if (vec_ok<InT>(x, s, dh)) {
      constexpr int N = Vec16<InT>::kN;
      const int rpw = 32 / (dh / N);
      const long long per_cta = 8LL * rpw * kRowsPerLane;
      const int grid = (int)((rows + per_cta - 1) / per_cta);
      if (dh == 128) quant_rows_vec_kernel<InT, 128><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, H, T, Tpad, q8, eq);
      else quant_rows_vec_kernel<InT, 64><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, H, T, Tpad, q8, eq);
      return launch_rc();
    }
    const int grid = (int)((rows + 7) / 8);
    quant_rows_kernel<InT><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, H, T, dh, Tpad, q8, eq);
    return launch_rc();
  });
}

int lssab8_quant_heads(const void* x, int dtype, int B, int H, int T, int dh, const int64_t* xs, int Tpad,
                       int8_t* q8, int32_t* eq, void* stream) {
  if (!x || !q8 || !eq || !shape_ok(B, H, H, T, dh) || Tpad < T || !strides_ok(xs, 4) || H > 65535 || B > 65535)
    return kErrArg;
  Strides4 s{xs[0], xs[1], xs[2], xs[3]};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    quant_head_kernel<InT><<<dim3(H, B), 256, 0, st>>>(static_cast<const InT*>(x), s, B, H, T, dh, Tpad, q8, eq);
    return launch_rc();
  });
}

int lssab8_quant_blocks(const void* x, int dtype, int B, int KVH, int T, int dh, const int64_t* xs, int Tpad,
                        int mode, int8_t* x8, int32_t* e, int32_t* e0, void* stream) {
  if (!x || !x8 || !e || !shape_ok(B, KVH, KVH, T, dh) || Tpad < tpad_of(T) || !strides_ok(xs, 4) || mode < 0 ||
      mode > 2 || (mode == 2 && !e0))
    return kErrArg;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  Strides4 s{xs[0], xs[1], xs[2], xs[3]};
  dim3 grid((T + 127) / 128, KVH, B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    if (vec_ok<InT>(x, s, dh) && Tpad == tpad_of(T)) {
      if (dh == 128)
        quant_blocks_vec_kernel<InT, 128><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, KVH, T, Tpad, mode, x8, e,
                                                                e0, ds->err);
      else
        quant_blocks_vec_kernel<InT, 64><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, KVH, T, Tpad, mode, x8, e,
                                                               e0, ds->err);
      return launch_rc();
    }
    quant_blocks_kernel<InT><<<grid, 256, 0, st>>>(static_cast<const InT*>(x), s, B, KVH, T, dh, Tpad, mode, x8, e, e0,
                                                   nullptr, ds->err);
    return launch_rc();
  });
}

int lssab8_quant_values_keyshift(const void* v, int dtype, int B, int KVH, int T, int dh, const int64_t* vs,
                                 int Tpad, int sink, int dmax, int8_t* v8, int32_t* ev, int32_t* ev0, int8_t* d8,
                                 void* stream) {
  if (!v || !v8 || !ev || !d8 || (sink && !ev0) || !shape_ok(B, KVH, KVH, T, dh) || Tpad < tpad_of(T) ||
      !strides_ok(vs, 4) || dmax < 1 || dmax > 16)
    return kErrArg;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  Strides4 s{vs[0], vs[1], vs[2], vs[3]};
  dim3 grid((T + 127) / 128, KVH, B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int mode = (sink && T > 1) ? 2 : 1;
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    quant_values_keyshift_kernel<InT><<<grid, 256, 0, st>>>(static_cast<const InT*>(v), s, B, KVH, T, dh, Tpad, mode,
                                                           dmax, v8, ev, ev0, d8, ds->err);
    return launch_rc();
  });
}

int lssab8_quant_keys_offset(const void* k, int dtype, int B, int KVH, int T, int dh, const int64_t* ks, int Tpad,
                             const float* mu, int8_t* k8, int32_t* ek, void* stream) {
  if (!k || !mu || !k8 || !ek || !shape_ok(B, KVH, KVH, T, dh) || Tpad < tpad_of(T) || !strides_ok(ks, 4))
    return kErrArg;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  Strides4 s{ks[0], ks[1], ks[2], ks[3]};
  dim3 grid((T + 127) / 128, KVH, B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    quant_blocks_kernel<InT><<<grid, 256, 0, st>>>(static_cast<const InT*>(k), s, B, KVH, T, dh, Tpad, 0, k8, ek,
                                                   nullptr, mu, ds->err);
    return launch_rc();
  });
}

int lssab8_prefill_lattice(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                           const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH, int T,
                           int dh, int Tpad, float* orow_scratch, void* out, int out_dtype, const int64_t* os,
                           void* stream) {
  if (Tpad != tpad_of(T)) return kErrArg;
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, ev0, B, H, KVH, 0, T, dh, orow_scratch, out, out_dtype, os,
                              stream);
}

int lssab8_prefill_lattice_general(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                   const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH,
                                   int T, int dh, int Tpad, int causal, const uint32_t* key_mask, float* out,
                                   const int64_t* os, void* stream) {
  if (Tpad != tpad_of(T) || !key_mask) return kErrArg;
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, ev0, B, H, KVH, 0, T, dh, nullptr, out, kF32, os, stream,
                              kWaitLimitNs, -1, 0, nullptr, 1, causal, key_mask);
}

int lssab8_prefill_lattice_keyshift(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                    const int8_t* v8, const int32_t* ev, const int32_t* ev0, const int8_t* d8, int B,
                                    int H, int KVH, int T, int dh, int Tpad, void* out, int out_dtype,
                                    const int64_t* os, void* stream) {
  if (Tpad != tpad_of(T) || !d8) return kErrArg;
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, ev0, B, H, KVH, 0, T, dh, nullptr, out, out_dtype, os, stream,
                              kWaitLimitNs, -1, 0, nullptr, 0, 1, nullptr, d8);
}

int lssab8_prefill_chunk_lattice(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                 const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH,
                                 int T0, int T, int dh, float* orow_scratch, void* out, int out_dtype,
                                 const int64_t* os, void* stream) {
  if (T0 < 0 || T0 % 128 != 0 || T0 >= T) return kErrArg;
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, ev0, B, H, KVH, T0, T, dh, orow_scratch, out, out_dtype, os,
                              stream);
}

size_t lssab8_prefill_workspace_size(int B, int H, int KVH, int T, int dh) {
  if (!shape_ok(B, H, KVH, T, dh)) return 0;
  return prefill_ws(B, H, KVH, T, dh).total;
}

}  // extern "C"

static int prefill_impl(const void* q, const void* k, const void* v, int dtype, int B, int H, int KVH, int T, int dh,
                        const int64_t* qs, const int64_t* ks, const int64_t* vs, int sink, void* out, int out_dtype,
                        const int64_t* os, void* workspace, size_t workspace_bytes, void* stream, int npeers,
                        void* const* peers) {
  if (!q || !k || !v || !out || !workspace || !shape_ok(B, H, KVH, T, dh)) return kErrArg;
  if (dh != 64 && dh != 128) return kErrUnsupported;
  const PrefillWs w = prefill_ws(B, H, KVH, T, dh);
  if (workspace_bytes < w.total) return kErrWorkspace;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const int Tpad = tpad_of(T);
  int8_t* q8 = reinterpret_cast<int8_t*>(base + w.q8);
  int32_t* eq = reinterpret_cast<int32_t*>(base + w.eq);
  int8_t* k8 = reinterpret_cast<int8_t*>(base + w.k8);
  int32_t* ek = reinterpret_cast<int32_t*>(base + w.ek);
  int8_t* v8 = reinterpret_cast<int8_t*>(base + w.v8);
  int32_t* ev = reinterpret_cast<int32_t*>(base + w.ev);
  int32_t* ev0 = reinterpret_cast<int32_t*>(base + w.ev0);
  int rc;
  const int vmode = sink ? (T > 1 ? 2 : 1) : 0;
  if (!strides_ok(qs, 4) || !strides_ok(ks, 4) || !strides_ok(vs, 4)) return kErrArg;
  DevState* ds = nullptr;
  if ((rc = dev_state(&ds))) return rc;
  const Strides4 sk{ks[0], ks[1], ks[2], ks[3]}, sv{vs[0], vs[1], vs[2], vs[3]};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = lssab8_quant_rows(q, dtype, B, H, T, dh, qs, Tpad, q8, eq, stream))) return rc;
  // K and V in one launch when both take the vectorised path
  rc = with_in_dtype(dtype, [&](auto tag) -> int {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    if (!vec_ok<InT>(k, sk, dh) || !vec_ok<InT>(v, sv, dh)) return -1;
    const int grid = 2 * (Tpad / 128) * KVH * B;
    auto kfn = (dh == 128) ? quant_kv_vec_kernel<InT, 128> : quant_kv_vec_kernel<InT, 64>;
    kfn<<<grid, 256, 0, st>>>(static_cast<const InT*>(k), sk, static_cast<const InT*>(v), sv, B, KVH, T, Tpad, vmode,
                              k8, ek, v8, ev, ev0, ds->err);
    return launch_rc();
  });
  if (rc > 0) return rc;
  if (rc < 0) {                                      // strided or unaligned inputs: the generic quantisers
    if ((rc = lssab8_quant_blocks(k, dtype, B, KVH, T, dh, ks, Tpad, 0, k8, ek, nullptr, stream))) return rc;
    if ((rc = lssab8_quant_blocks(v, dtype, B, KVH, T, dh, vs, Tpad, vmode, v8, ev, ev0, stream))) return rc;
  }
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, (sink && T > 1) ? ev0 : nullptr, B, H, KVH, 0, T, dh, nullptr,
                              out, out_dtype, os, stream, kWaitLimitNs, -1, npeers, peers);
}

extern "C" {

int lssab8_prefill(const void* q, const void* k, const void* v, int dtype, int B, int H, int KVH, int T, int dh,
                   const int64_t* qs, const int64_t* ks, const int64_t* vs, int sink, void* out, int out_dtype,
                   const int64_t* os, void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_impl(q, k, v, dtype, B, H, KVH, T, dh, qs, ks, vs, sink, out, out_dtype, os, workspace,
                      workspace_bytes, stream, 0, nullptr);
}

int lssab8_prefill_peers(const void* q, const void* k, const void* v, int dtype, int B, int H, int KVH, int T, int dh,
                         const int64_t* qs, const int64_t* ks, const int64_t* vs, int sink, void* out, int out_dtype,
                         const int64_t* os, void* const* peer_out, int npeers, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (npeers < 0 || npeers > kMaxPeers) return kErrArg;
  return prefill_impl(q, k, v, dtype, B, H, KVH, T, dh, qs, ks, vs, sink, out, out_dtype, os, workspace,
                      workspace_bytes, stream, npeers, peer_out);
}

// ------------------------------------------------------------ peer buffers (CUDA IPC)
static PFN_cuMemGetAddressRange_v3020 g_range = nullptr;

static int get_range_fn() {
  static std::once_flag once;
  static int rc = kOk;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      rc = kErrCuda;
      return;
    }
    g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  return rc;
}

int lssab8_peer_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return kErrArg;
  if (get_range_fn() != kOk) return kErrCuda;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return kErrArg;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return kErrCuda;
  std::memcpy(handle, &h, sizeof h);
  *offset = (uint64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return kOk;
}

int lssab8_peer_import(const void* handle, uint64_t offset, int owner_device, void** ptr) {
  if (!handle || !ptr) return kErrArg;
  int dev = 0, can = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  if (owner_device == dev) return kErrArg;
  if (cudaDeviceCanAccessPeer(&can, dev, owner_device) != cudaSuccess) return kErrCuda;
  if (!can) return kErrUnsupported;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return kErrCuda;
  *ptr = static_cast<uint8_t*>(base) + offset;
  return kOk;
}

int lssab8_peer_close(void* ptr, uint64_t offset) {
  if (!ptr) return kErrArg;
  return cuda_rc(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset));
}

int lssab8_peer_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
                       void* stream) {
  if (!dst || !src || width == 0 || width > dpitch || width > spitch) return kErrArg;
  if (height == 0) return kOk;
  return cuda_rc(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDeviceToDevice,
                                   static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

// the vectorised lattice writer applies when channels are contiguous, dh is 64 or 128, and every
// row start is 16-byte aligned (base, the row / head / page strides and, for a contiguous source,
// each sequence offset a multiple of 16 bytes)
static int kv_lattice_launch(const void* k, const void* v, int dtype, int B, int KVH, int dh, const int32_t* seq_lens,
                             const int32_t* start_lens, const int64_t* seq_off, int64_t st, int64_t sg, int64_t sc,
                             const int32_t* src_bt, int64_t src_ps, const int32_t* block_table, int max_pages,
                             int max_blocks, int num_pages, int sink, int8_t* k8p, int8_t* v8p, int32_t* ek,
                             int32_t* ev, int32_t* ev0, int* err, cudaStream_t s, bool* done) {
  *done = false;
  if ((dh != 64 && dh != 128) || sc != 1) return kOk;
  return with_in_dtype(dtype, [&](auto tag) -> int {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    const long long e = (long long)sizeof(InT);
    if ((reinterpret_cast<uintptr_t>(k) & 15) || (reinterpret_cast<uintptr_t>(v) & 15) || (st * e) % 16 ||
        (sg * e) % 16 || (src_bt && (src_ps * e) % 16))
      return kOk;
    if (B > 32767) return kOk;
    dim3 grid(max_blocks, KVH, 2 * B);                  // K and V blocks in separate CTAs
    const int vmode = sink ? 2 : 0;
    auto kfn = dh == 128 ? kv_lattice_kernel<InT, 128> : kv_lattice_kernel<InT, 64>;
    const int nt = dh == 128 ? KvLattice<InT, 128>::kThreads : KvLattice<InT, 64>::kThreads;
    kfn<<<grid, nt, 0, s>>>(static_cast<const InT*>(k), static_cast<const InT*>(v),
                             reinterpret_cast<const long long*>(seq_off), st, sg, src_bt, src_ps, B, KVH, seq_lens,
                             start_lens, block_table, max_pages, max_blocks, num_pages, vmode, k8p, v8p, ek, ev, ev0,
                             err);
    *done = true;
    return launch_rc();
  });
}

extern "C" {

int lssab8_kv_append(const void* k, const void* v, int dtype, int B, int KVH, int dh, const int32_t* seq_lens,
                     const int32_t* start_lens, const int64_t* seq_off, int64_t st, int64_t sg, const int32_t* src_block_table,
                     int64_t src_page_stride, const int32_t* block_table, int max_pages, int max_blocks, int num_pages,
                     int sink, int8_t* k8p, int8_t* v8p, int32_t* ek, int32_t* ev, int32_t* ev0, void* stream) {
  if (!k || !v || !seq_lens || !start_lens || (!seq_off && !src_block_table) || !block_table || !k8p || !v8p || !ek ||
      !ev || (sink && !ev0) || B <= 0 || KVH <= 0 || max_pages <= 0 || max_blocks <= 0 || num_pages <= 0 || st < 0 ||
      sg < 0 || src_page_stride < 0 || max_pages < max_blocks * 8 - 7)
    return kErrArg;
  if (dh != 64 && dh != 128) return kErrUnsupported;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  bool done = false;
  rc = kv_lattice_launch(k, v, dtype, B, KVH, dh, seq_lens, start_lens, seq_off, st, sg, 1, src_block_table,
                         src_page_stride, block_table, max_pages, max_blocks, num_pages, sink, k8p, v8p, ek, ev, ev0,
                         ds->err, static_cast<cudaStream_t>(stream), &done);
  if (rc) return rc;
  return done ? kOk : kErrArg;                       // unaligned rows: the append needs 16-byte rows
}

int lssab8_decode_prep_kv(const void* k, const void* v, int dtype, int B, int KVH, int dh, const int32_t* seq_lens,
                          const int64_t* seq_off, int64_t st, int64_t sg, int64_t sc, const int32_t* block_table,
                          int max_pages, int max_blocks, int num_pages, int sink, int8_t* k8p, int8_t* v8p,
                          int32_t* ek, int32_t* ev, int32_t* ev0, void* stream) {
  if (!k || !v || !seq_lens || !seq_off || !block_table || !k8p || !v8p || !ek || !ev || (sink && !ev0) || B <= 0 ||
      KVH <= 0 || dh <= 0 || dh > 256 || max_pages <= 0 || max_blocks <= 0 || num_pages <= 0 || st < 0 || sg < 0 ||
      sc < 0 || max_pages < max_blocks * 8 - 7)
    return kErrArg;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  dim3 grid(max_blocks, KVH, B);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int vmode = sink ? 2 : 0;
  bool done = false;
  if ((rc = kv_lattice_launch(k, v, dtype, B, KVH, dh, seq_lens, nullptr, seq_off, st, sg, sc, nullptr, 0,
                              block_table, max_pages, max_blocks, num_pages, sink, k8p, v8p, ek, ev, ev0, ds->err, s,
                              &done)))
    return rc;
  if (done) return kOk;
  return with_in_dtype(dtype, [&](auto tag) {
    using InT = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    decode_prep_kernel<InT><<<grid, 256, 0, s>>>(static_cast<const InT*>(k), static_cast<const InT*>(v),
                                                 reinterpret_cast<const long long*>(seq_off), st, sg, sc, B, KVH, dh,
                                                 seq_lens, block_table, max_pages, max_blocks, num_pages, vmode, k8p,
                                                 v8p, ek, ev, ev0, ds->err);
    return launch_rc();
  });
}

size_t lssab8_decode_workspace_size(int B, int H, int KVH, int dh, int max_blocks) {
  if (B <= 0 || H <= 0 || KVH <= 0 || H % KVH || dh <= 0 || max_blocks <= 0) return 0;
  return decode_ws(B, H, KVH, dh, max_blocks).total;
}

int lssab8_decode(const void* q, int dtype, const int64_t* qs, int B, int H, int KVH, int dh, const int32_t* seq_lens,
                  const int32_t* block_table, int max_pages, int num_pages, const int8_t* k8p, const int8_t* v8p,
                  const int32_t* ek, const int32_t* ev, const int32_t* ev0, int max_blocks, int split_blocks, int sink,
                  void* out, int out_dtype, const int64_t* os, void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !seq_lens || !block_table || !k8p || !v8p || !ek || !ev || (sink && !ev0) || !out || !workspace ||
      !strides_ok(qs, 3) || !strides_ok(os, 3) || B <= 0 || H <= 0 || KVH <= 0 || H % KVH || max_blocks <= 0 ||
      split_blocks <= 0 || max_pages <= 0 || num_pages <= 0)
    return kErrArg;
  if ((dh != 64 && dh != 128) || H / KVH > 8) return kErrUnsupported;
  const DecodeWs w = decode_ws(B, H, KVH, dh, max_blocks);
  if (workspace_bytes < w.total) return kErrWorkspace;
  DevState* ds = nullptr;
  int rc = dev_state(&ds);
  if (rc) return rc;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  int8_t* q8 = reinterpret_cast<int8_t*>(base + w.q8);
  int32_t* eq = reinterpret_cast<int32_t*>(base + w.eq);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t q4[4] = {qs[0], qs[1], 0, qs[2]};
  // (the ticket reset and the plan come first so the query quantiser directly precedes the
  // decode kernel, which may then start under programmatic dependent launch)
  if (dh == 128) {                                   // the live-block plan; it also zeroes the tickets
    decode_plan_kernel<<<1, kPlanThreads, 0, s>>>(seq_lens, B, max_blocks, max_pages,
                                                  reinterpret_cast<int*>(base + w.blk_off),
                                                  reinterpret_cast<int*>(base + w.order),
                                                  reinterpret_cast<unsigned int*>(base + w.tickets), B * KVH, ds->err);
    if ((rc = launch_rc())) return rc;
  } else if (cudaMemsetAsync(base + w.tickets, 0, (size_t)B * KVH * 4, s) != cudaSuccess) {
    return kErrCuda;
  }
  if ((rc = dh == 128 ? quant_queries_pdl(q, dtype, B, H, dh, q4, q8, eq, s)
                      : lssab8_quant_rows(q, dtype, B, H, 1, dh, q4, 1, q8, eq, stream)))
    return rc;
  DecodeArgs a{};
  a.B = B; a.H = H; a.KVH = KVH; a.dh = dh; a.group = H / KVH; a.max_blocks = max_blocks; a.max_pages = max_pages;
  a.split_blocks = split_blocks; a.num_pages = num_pages; a.seq_lens = seq_lens; a.block_table = block_table;
  a.k8p = k8p; a.v8p = v8p; a.ek = ek; a.ev = ev; a.ev0 = sink ? ev0 : nullptr; a.q8 = q8; a.eq = eq;
  a.partA = reinterpret_cast<int32_t*>(base + w.partA);
  a.partM = reinterpret_cast<int4*>(base + w.partM);
  a.tickets = reinterpret_cast<unsigned int*>(base + w.tickets);
  a.blk_off = reinterpret_cast<int*>(base + w.blk_off);
  a.order = reinterpret_cast<int*>(base + w.order);
  a.out = out; a.os0 = os[0]; a.os1 = os[1]; a.os2 = os[2];
  a.gbase = gbase_of(dh);
  a.err = ds->err;
  const int max_splits = (max_blocks + split_blocks - 1) / split_blocks;
  if (dh == 128) return sink ? launch_decode_tc_out<true>(out_dtype, a, max_splits, ds->num_sms, s)
                             : launch_decode_tc_out<false>(out_dtype, a, max_splits, ds->num_sms, s);
  return sink ? launch_decode_out<64, true>(out_dtype, a, max_splits, s)
              : launch_decode_out<64, false>(out_dtype, a, max_splits, s);
}

// ------------------------------------------------------------ allocation-free decode
// The fixed scratch of lssab8_decode_noalloc (see include/lssab8.h): a file-scope device array.
// In host code its name is only a host-side stand-in, never a device address; the device address
// is looked up once per device with cudaGetSymbolAddress, with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LSSAB8_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrCuda;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return kErrCuda;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}
}  // namespace

int lssab8_decode_noalloc(const void* q, int dtype, const int64_t* qs, int B, int H, int KVH, int dh,
                          const int32_t* seq_lens, const int32_t* block_table, int max_pages, int num_pages,
                          const int8_t* k8p, const int8_t* v8p, const int32_t* ek, const int32_t* ev,
                          const int32_t* ev0, int max_blocks, int split_blocks, int sink, void* out, int out_dtype,
                          const int64_t* os, void* stream) {
  if (!q || !seq_lens || !block_table || !k8p || !v8p || !ek || !ev || (sink && !ev0) || !out ||
      !strides_ok(qs, 3) || !strides_ok(os, 3) || B <= 0 || H <= 0 || KVH <= 0 || H % KVH || max_blocks <= 0 ||
      split_blocks <= 0 || max_pages <= 0 || num_pages <= 0)
    return kErrArg;
  if ((dh != 64 && dh != 128) || H / KVH > 8) return kErrUnsupported;
  const DecodeWs w = decode_ws(B, H, KVH, dh, max_blocks);
  if (w.total - 256 > (size_t)LSSAB8_NOALLOC_SCRATCH_BYTES) return LSSAB8_ESCRATCH;   // base is 256-aligned
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  DevState* ds = nullptr;
  if ((rc = dev_state(&ds))) return rc;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  int8_t* q8 = reinterpret_cast<int8_t*>(base + w.q8);
  int32_t* eq = reinterpret_cast<int32_t*>(base + w.eq);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t q4[4] = {qs[0], qs[1], 0, qs[2]};
  // the tickets must start at zero (the buffer keeps whatever the previous call left); the reset
  // and the plan come first, as in lssab8_decode, so the query quantiser directly precedes the
  // decode kernel
  if (dh == 128) {                                   // the live-block plan; it also zeroes the tickets
    decode_plan_kernel<<<1, kPlanThreads, 0, s>>>(seq_lens, B, max_blocks, max_pages,
                                                  reinterpret_cast<int*>(base + w.blk_off),
                                                  reinterpret_cast<int*>(base + w.order),
                                                  reinterpret_cast<unsigned int*>(base + w.tickets), B * KVH, ds->err);
    if ((rc = launch_rc())) return rc;
  } else if (cudaMemsetAsync(base + w.tickets, 0, (size_t)B * KVH * 4, s) != cudaSuccess) {
    return kErrCuda;
  }
  if ((rc = dh == 128 ? quant_queries_pdl(q, dtype, B, H, dh, q4, q8, eq, s)
                      : lssab8_quant_rows(q, dtype, B, H, 1, dh, q4, 1, q8, eq, stream)))
    return rc;
  DecodeArgs a{};
  a.B = B; a.H = H; a.KVH = KVH; a.dh = dh; a.group = H / KVH; a.max_blocks = max_blocks; a.max_pages = max_pages;
  a.split_blocks = split_blocks; a.num_pages = num_pages; a.seq_lens = seq_lens; a.block_table = block_table;
  a.k8p = k8p; a.v8p = v8p; a.ek = ek; a.ev = ev; a.ev0 = sink ? ev0 : nullptr; a.q8 = q8; a.eq = eq;
  a.partA = reinterpret_cast<int32_t*>(base + w.partA);
  a.partM = reinterpret_cast<int4*>(base + w.partM);
  a.tickets = reinterpret_cast<unsigned int*>(base + w.tickets);
  a.blk_off = reinterpret_cast<int*>(base + w.blk_off);
  a.order = reinterpret_cast<int*>(base + w.order);
  a.out = out; a.os0 = os[0]; a.os1 = os[1]; a.os2 = os[2];
  a.gbase = gbase_of(dh);
  a.err = ds->err;
  const int max_splits = (max_blocks + split_blocks - 1) / split_blocks;
  if (dh == 128) return sink ? launch_decode_tc_out<true>(out_dtype, a, max_splits, ds->num_sms, s)
                             : launch_decode_tc_out<false>(out_dtype, a, max_splits, ds->num_sms, s);
  return sink ? launch_decode_out<64, true>(out_dtype, a, max_splits, s)
              : launch_decode_out<64, false>(out_dtype, a, max_splits, s);
}

int lssab8_selftest_timeout(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                            const int8_t* v8, const int32_t* ev, int B, int H, int KVH, int T, int dh,
                            int withhold_block, int wait_us, void* out, const int64_t* os, void* stream) {
  if (withhold_block < 0 || wait_us <= 0 || wait_us > 2000000) return kErrArg;
  return prefill_lattice_impl(q8, eq, k8, ek, v8, ev, nullptr, B, H, KVH, 0, T, dh, nullptr, out, kF32, os, stream,
                              (uint64_t)wait_us * 1000ull, withhold_block);
}

int lssab8_selftest_div(const float* y, const float* l, long long n, float* out, void* stream) {
  if (!y || !l || !out || n < 0) return kErrArg;
  if (n == 0) return kOk;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
  selftest_div_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, l, n, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int lssab8_selftest_rescale(const float* x, const int32_t* D, long long npairs, float* out, void* stream) {
  if (!x || !D || !out || npairs < 0) return kErrArg;
  if (npairs == 0) return kOk;
  const int blocks = (int)std::min<long long>((npairs + 255) / 256, 148LL * 16);
  selftest_rescale_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, D, npairs, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // extern "C"
