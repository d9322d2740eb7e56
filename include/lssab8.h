/*
 * lssab8.h -- C ABI of liblssab8_b200.so: LSSA-B8 / B9.1 contract attention on B200 (sm_100a).
 *
 * Plain pointers and sizes only.  All device pointers live on the CUDA device that is current
 * when the call is made; every call is asynchronous on `stream` (a cudaStream_t, NULL = the
 * legacy default stream) and never allocates device memory: buffers, including workspaces,
 * belong to the caller.  Every entry point returns 0 on success or a LSSAB8_E* code; no C++
 * exception crosses the ABI.  Calls on different streams are independent (thread-safe per
 * stream); the device error word is per device.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   reference/lssab8_torch.py:103-272  make_lssab8_long_attn(...) -> attn(module, q, k, v, mask)
 *   reference/lssab8_torch.py:275-281  make_lssab8_attn
 *   reference/lssab9_torch.py:68-327   make_lssab9_long_attn(..., sink_alone=True)
 *   reference/lssab8_golden.py:341-346 lssab8_attention;  :200-338 lssab8_core
 *   reference/lssab8_golden.py:350-394 lssab8_row_segments (split-KV decode structure)
 *   reference/lssab_golden.py:214-235  lssab_quantize (PREP);  reference/t10_attn.py:40-48 quant_rows;
 *   reference/lssab_torch.py:62-85     quant_pow2_blocks;  reference/lssab9_torch.py:46-65,121-132
 *
 * Strides are in ELEMENTS (not bytes), int64[4] unless stated.
 * dtype codes: 0 = float32, 1 = float16, 2 = bfloat16.
 */
#ifndef LSSAB8_H
#define LSSAB8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LSSAB8_OK = 0,
  LSSAB8_EARG = 1,          /* bad shape, stride, dtype or null pointer                      */
  LSSAB8_EUNSUPPORTED = 2,  /* a contract-valid input these kernels do not cover (e.g. dh)    */
  LSSAB8_ECUDA = 3,         /* a CUDA runtime/driver call failed                              */
  LSSAB8_EWORKSPACE = 4,    /* the caller's workspace is smaller than *_workspace_size()      */
  LSSAB8_EDEVICE = 5,       /* the device error word is nonzero (lssab8_device_errors)        */
  LSSAB8_ESCRATCH = 6       /* lssab8_decode_noalloc: the problem needs more scratch than the
                               library's fixed buffer (LSSAB8_NOALLOC_SCRATCH_BYTES)            */
};

/* Size of the fixed device scratch buffer behind lssab8_decode_noalloc (48 MiB). */
#define LSSAB8_NOALLOC_SCRATCH_BYTES (48u << 20)

/* device error bits (OR-accumulated by kernels; read with lssab8_device_errors) */
enum {
  LSSAB8_DEV_EV_RANGE = 1,  /* e_v outside [-32, 40]: reference/lssab9_torch.py:158 assert    */
  LSSAB8_DEV_TIMEOUT = 2,   /* a bounded pipeline wait gave up                                */
  LSSAB8_DEV_BAD_PAGE = 4,  /* a block-table entry outside [0, num_pages)                     */
  LSSAB8_DEV_ALIGN = 8      /* lssab8_kv_append: a source row not on a 16-byte boundary        */
};

/* Library identity: writes "lssab8-b200 <version> T2=<sha256 of the T2 csv>" (NUL-terminated)
 * into buf.  The digest is recomputed from the table compiled into the device code, so it
 * pins the constants (reference/lssab8_golden.py:117-128).  Returns LSSAB8_EARG if buflen is
 * too small (needs 128 bytes). */
int lssab8_version(char* buf, int buflen);

/* Human-readable text for a status code. */
const char* lssab8_strerror(int code);

/* Synchronise `stream`, store the current device's error word in *bits, clear it if `clear`. */
int lssab8_device_errors(int clear, void* stream, int* bits);

/* ---------------------------------------------------------------- PREP (P1 / P2 / P3) */

/* P1: per-(row) pow2 quantiser.  x [B, H, T, dh] (strides xs) -> q8 [B, H, Tpad, dh] int8 and
 * eq [B, H, Tpad] int32, rows >= T zero.  reference/t10_attn.py:40-48. */
int lssab8_quant_rows(const void* x, int dtype, int B, int H, int T, int dh, const int64_t* xs, int Tpad,
                      int8_t* q8, int32_t* eq, void* stream);

/* P1 with one exponent per head (the golden's q_exp_mode "head", reference/lssab_golden.py:
 * 230-232): the row rule applied to all T rows and dh channels of a head at once.  Same layout
 * as lssab8_quant_rows; eq[b, h, t] holds the head's exponent for every t < T. */
int lssab8_quant_heads(const void* x, int dtype, int B, int H, int T, int dh, const int64_t* xs, int Tpad,
                       int8_t* q8, int32_t* eq, void* stream);

/* P2/P3: per-(128-key block, kv head) quantiser.  x [B, KVH, T, dh] -> x8 [B, KVH, Tpad, dh],
 * e [B, KVH, ceil(T/128)], e0 [B, KVH] (mode 2 only).  mode 0 = B8 grid
 * (reference/lssab_torch.py:62-85), 1 = B9 value grid (reference/lssab9_torch.py:46-65,158),
 * 2 = B9.1 sink_alone value grid (reference/lssab9_torch.py:124-132). */
int lssab8_quant_blocks(const void* x, int dtype, int B, int KVH, int T, int dh, const int64_t* xs, int Tpad,
                        int mode, int8_t* x8, int32_t* e, int32_t* e0, void* stream);

/* B9.3 value quantiser (v_keyshift = dmax in [1, 16]; reference/lssab9_golden.py:37-70,
 * reference/lssab9_torch.py:145-153): the B9 value grid per 128-key block (e_v clamped to
 * [-32, 48], LSSAB8_DEV_EV_RANGE when outside [-32, 40]; sink = 1 and T > 1: key 0 alone on ev0 as in
 * mode 2 of lssab8_quant_blocks), then key j on the finer grid e_tok + d_j with
 * d_j = clamp(e_j - e_tok, 0, dmax), e_j the key row's own exponent on the B9 grid and e_tok the
 * exponent its block gives it.  v8 [B, KVH, Tpad, dh], ev [B, KVH, nblk], ev0 [B, KVH] (sink),
 * d8 [B, KVH, Tpad] int8 (d_j; padding keys 0). */
int lssab8_quant_values_keyshift(const void* v, int dtype, int B, int KVH, int T, int dh, const int64_t* vs,
                                 int Tpad, int sink, int dmax, int8_t* v8, int32_t* ev, int32_t* ev0, int8_t* d8,
                                 void* stream);

/* P2 with the key offset: k' = fl(f32(k) - mu[g, c]) in binary32, then the B8 block quantiser
 * (mode 0) on k'.  mu [KVH, dh] float32 on the device, one offset per kv head and channel (the
 * reference's per-layer mu[layer], reference/lssab8_torch.py:143-144, reference/lssab_golden.py:
 * 214-221).  k8/ek as lssab8_quant_blocks writes them. */
int lssab8_quant_keys_offset(const void* k, int dtype, int B, int KVH, int T, int dh, const int64_t* ks, int Tpad,
                             const float* mu, int8_t* k8, int32_t* ek, void* stream);

/* --------------------------------------------------------------------------- prefill */

/* Causal GQA prefill on a prepared lattice (the output of the two quantisers with
 * Tpad = 128*ceil(T/128)).  out[b, t, h, c] at out + b*os[0] + t*os[1] + h*os[2] + c*os[3] in
 * out_dtype.  ev0 = NULL: sink off (B8); non-NULL: B9.1 sink_alone.  dh in {64, 128}.
 * orow_scratch: unused and may be NULL (rows spanning more than one 32-block fold segment keep
 * their row accumulator in tensor memory); the parameter stays for ABI stability.
 * The fold of reference/lssab8_torch.py:164-271 / reference/lssab9_torch.py:176-326. */
int lssab8_prefill_lattice(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                           const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH, int T,
                           int dh, int Tpad, float* orow_scratch, void* out, int out_dtype, const int64_t* os,
                           void* stream);

/* The general form of lssab8_prefill_lattice, for the golden entry points
 * (reference/lssab8_golden.py:341-346 lssab8_attention(..., causal, key_valid),
 * reference/lssab9_golden.py:254-259 lssab9_attention): causal = 0 lets every query row see
 * every key; key_mask [B, Tpad / 32] uint32 words (bit j % 32 of word j / 32 of batch element b
 * set: key j is visible to every row of b; bits of keys >= T must be clear) is required.  A row
 * that sees no key of a block skips it, a row that sees no key at all yields 0, exactly as the
 * golden's visibility rule (reference/lssab8_golden.py:241-247).  out float32 [b, t, h, c]. */
int lssab8_prefill_lattice_general(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                   const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH,
                                   int T, int dh, int Tpad, int causal, const uint32_t* key_mask, float* out,
                                   const int64_t* os, void* stream);

/* Causal prefill with B9.3 (v_keyshift): as lssab8_prefill_lattice on a lattice whose values and
 * per-key shifts d8 [B, KVH, Tpad] come from lssab8_quant_values_keyshift; key j's PV weight is
 * eh_j >> d_j while l_b sums the unshifted eh_j (reference/lssab9_golden.py:179-186).  out_dtype
 * float32 or bfloat16. */
int lssab8_prefill_lattice_keyshift(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                    const int8_t* v8, const int32_t* ev, const int32_t* ev0, const int8_t* d8, int B,
                                    int H, int KVH, int T, int dh, int Tpad, void* out, int out_dtype,
                                    const int64_t* os, void* stream);

/* Block-aligned chunked prefill on an append-only lattice: query rows [T0, T) of a sequence
 * (T0 a multiple of 128) against keys [0, T).  q8/eq hold the chunk's rows only, quantised per
 * row as by lssab8_quant_rows ([B, H, Tq, dh] / [B, H, Tq], Tq = 128*ceil((T - T0)/128));
 * k8/v8/ek/ev/ev0 hold the lattice of the whole prefix [0, T) as lssab8_quant_blocks writes it
 * (Tpad = 128*ceil(T/128)), so blocks completed by earlier chunks are reused as they are; out
 * holds the chunk's T - T0 rows (row t of the sequence at t - T0); orow_scratch unused (NULL).  No counterpart entry point in
 * the reference: its 128-aligned chunk invariance (reference/lssab8_selftest.py:292-317) makes
 * the result bit-identical to rows [T0, T) of the whole prefill of length T. */
int lssab8_prefill_chunk_lattice(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                                 const int8_t* v8, const int32_t* ev, const int32_t* ev0, int B, int H, int KVH,
                                 int T0, int T, int dh, float* orow_scratch, void* out, int out_dtype,
                                 const int64_t* os, void* stream);

/* Bytes of workspace lssab8_prefill needs for this shape. */
size_t lssab8_prefill_workspace_size(int B, int H, int KVH, int T, int dh);

/* The whole drop-in: PREP + prefill.  q [B, H, T, dh], k/v [B, KVH, T, dh] in `dtype` with
 * strides qs/ks/vs; out as in lssab8_prefill_lattice.  sink = 0: LSSA-B8
 * (reference/lssab8_torch.py:134-271 per batch element); sink = 1: LSSA-B9.1 sink_alone
 * (reference/lssab9_torch.py:109-326 with sink_alone=True). */
int lssab8_prefill(const void* q, const void* k, const void* v, int dtype, int B, int H, int KVH, int T, int dh,
                   const int64_t* qs, const int64_t* ks, const int64_t* vs, int sink, void* out, int out_dtype,
                   const int64_t* os, void* workspace, size_t workspace_bytes, void* stream);

/* The sharded form of lssab8_prefill, with the output gather fused into the kernel.  No
 * reference counterpart: the reference has no multi-GPU attention; the split is the one the
 * contract allows (every row is an independent recurrence, so kv-head groups shard with no
 * arithmetic across ranks).  Rank r of n runs lssab8_prefill on its kv heads and their query
 * heads, writing its rows into its own output buffer out (strides os) AND, with the same element
 * offsets, into each of the npeers (<= 7) addresses peer_out[i]: the other ranks' output buffers
 * mapped into this process (lssab8_peer_import), each congruent to out modulo 16 bytes.  The
 * stores go over NVLink as the tiles finish; each CTA ends with a system-scope fence, so once
 * the kernel has completed on every rank (a barrier ordered after it on each rank's stream) every
 * rank's buffer holds every rank's heads.  The caller also orders a barrier before the call, so
 * that no rank writes into a buffer its owner is still reading. */
int lssab8_prefill_peers(const void* q, const void* k, const void* v, int dtype, int B, int H, int KVH, int T, int dh,
                         const int64_t* qs, const int64_t* ks, const int64_t* vs, int sink, void* out, int out_dtype,
                         const int64_t* os, void* const* peer_out, int npeers, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Peer buffers for lssab8_prefill_peers (CUDA IPC; no reference counterpart).
 * lssab8_peer_export: the 64-byte IPC handle of the device allocation holding ptr (written to
 *   handle) and ptr's byte offset in it.
 * lssab8_peer_import: maps another process's exported buffer, owned by CUDA device owner_device
 *   (an ordinal of this process), into this process with peer access from the current device
 *   enabled, and returns the address of the exported ptr in *ptr.  LSSAB8_EUNSUPPORTED when the
 *   current device cannot reach owner_device by peer access.
 * lssab8_peer_close: unmaps an address lssab8_peer_import returned (with its offset). */
int lssab8_peer_export(const void* ptr, void* handle, uint64_t* offset);
int lssab8_peer_import(const void* handle, uint64_t offset, int owner_device, void** ptr);
int lssab8_peer_close(void* ptr, uint64_t offset);

/* The sharded prefill's gather on the copy engines (no SM time): copies a height x width-byte
 * slab, rows dpitch / spitch bytes apart, from this GPU's output to a peer's buffer mapped by
 * lssab8_peer_import (cudaMemcpy2DAsync on `stream`, device to device over NVLink).  A rank's
 * head slice of out [B, T, H, dh] is such a slab: width h*dh*e bytes, pitch H*dh*e, B*T rows. */
int lssab8_peer_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
                       void* stream);

/* ---------------------------------------------------------------------------- decode */

/* Paged int8 lattice writer.  Sequence b has seq_lens[b] tokens; token t, kv head g, channel c
 * of K is read at k + seq_off[b] + t*st + g*sg + c*sc (same for v).  Pages hold 16 keys:
 * k8p [num_pages, KVH, 16, dh], v8p [num_pages, KVH, dh, 16] (values transposed per page);
 * block_table [B, max_pages] maps logical page -> physical page.  ek/ev [B, KVH, max_blocks]
 * int32 per logical 128-key block, ev0 [B, KVH] (sink only; may be NULL when sink = 0).
 * Block exponents cover the block's present rows only (reference/lssab_torch.py:62-85). */
int lssab8_decode_prep_kv(const void* k, const void* v, int dtype, int B, int KVH, int dh, const int32_t* seq_lens,
                          const int64_t* seq_off, int64_t st, int64_t sg, int64_t sc, const int32_t* block_table,
                          int max_pages, int max_blocks, int num_pages, int sink, int8_t* k8p, int8_t* v8p,
                          int32_t* ek, int32_t* ev, int32_t* ev0, void* stream);

/* Append to the paged int8 lattice (the engine's per-step lattice update; no counterpart entry
 * point in the reference, whose engine fuses it into decode: docs/contract/
 * BLOCK_EXPONENT_VARIANT.md:53-55, 212-215, docs/SPEC.md:2396-2412).  Sequence b grew from
 * start_lens[b] to seq_lens[b] tokens; the blocks complete before the append (index <
 * start_lens[b] / 128) are left untouched -- their values and exponents never change -- and the
 * open block and every new block are (re)quantised over their present rows from the caller's
 * float cache, so the lattice equals lssab8_decode_prep_kv's over all seq_lens[b] tokens bit for
 * bit.  The float cache: token t, kv head g, channel c at k + seq_off[b] + t*st + g*sg + c
 * (src_block_table NULL), or, for a paged cache, at
 * k + src_block_table[b, t / 16] * src_page_stride + (t % 16) * st + g*sg + c
 * (src_block_table [B, max_pages], 16-token pages, e.g. the same table as the lattice's; the
 * cache holds at least num_pages pages, and a source page id outside [0, num_pages) sets the
 * bad-page device error and the page is not read).
 * Channels contiguous, every row 16-byte aligned, dh in {64, 128}; lattice arguments as in
 * lssab8_decode_prep_kv. */
int lssab8_kv_append(const void* k, const void* v, int dtype, int B, int KVH, int dh, const int32_t* seq_lens,
                     const int32_t* start_lens, const int64_t* seq_off, int64_t st, int64_t sg, const int32_t* src_block_table,
                     int64_t src_page_stride, const int32_t* block_table, int max_pages, int max_blocks, int num_pages,
                     int sink, int8_t* k8p, int8_t* v8p, int32_t* ek, int32_t* ev, int32_t* ev0, void* stream);

/* Bytes of workspace lssab8_decode needs. */
size_t lssab8_decode_workspace_size(int B, int H, int KVH, int dh, int max_blocks);

/* Split-KV decode: one new query row per sequence, q [B, H, dh] (strides qs[0..2]), attending to
 * all seq_lens[b] keys of the lattice (the new token's own key is the last one).  Every
 * 128-key block yields exact block partials in the workspace, and a refold folds them in
 * ascending order (reference/lssab8_golden.py:350-394): at dh 128 a separate refold kernel runs
 * after the streaming kernel; at dh 64 the last split of each (sequence, kv head) to finish does
 * it.  split_blocks (blocks per split) changes no bit.  Equals row L-1 of the prefill
 * bit for bit (reference/lssab8_selftest.py:320-336).  out[b, h, c] at out + b*os[0] + h*os[1]
 * + c*os[2].  H/KVH <= 8, dh in {64, 128}. */
int lssab8_decode(const void* q, int dtype, const int64_t* qs, int B, int H, int KVH, int dh, const int32_t* seq_lens,
                  const int32_t* block_table, int max_pages, int num_pages, const int8_t* k8p, const int8_t* v8p,
                  const int32_t* ek, const int32_t* ev, const int32_t* ev0, int max_blocks, int split_blocks, int sink,
                  void* out, int out_dtype, const int64_t* os, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free decode.  No counterpart in the reference: it exists for hosts that cannot
 * hand this library a workspace.  Some engines plan all device memory up front and give each
 * attention call only its inputs and outputs; some plugin hosts own every device allocation and
 * expose no allocator to the plugin.  Such callers cannot call cudaMalloc for the split-KV
 * partials that lssab8_decode needs, so this entry point takes the same arguments as
 * lssab8_decode minus the workspace and uses a fixed scratch buffer of
 * LSSAB8_NOALLOC_SCRATCH_BYTES that the library holds in device memory on every GPU it is loaded
 * on, until the process exits.  It allocates nothing.
 *   - The call is refused with LSSAB8_ESCRATCH, launching nothing, exactly when
 *     lssab8_decode_workspace_size(B, H, KVH, dh, max_blocks) - 256 > LSSAB8_NOALLOC_SCRATCH_BYTES
 *     (the workspace size includes 256 bytes of alignment slack, which the 256-aligned buffer
 *     does not need).
 *   - The first call on a device looks up the buffer's device address for that device (with
 *     that device current); make that first call before any stream capture.
 *   - Every call on a device shares the one buffer: calls that can overlap on the GPU (other
 *     streams, other host threads) race and corrupt each other's results; serialise them.
 * Results are bit-identical to lssab8_decode's. */
int lssab8_decode_noalloc(const void* q, int dtype, const int64_t* qs, int B, int H, int KVH, int dh,
                          const int32_t* seq_lens, const int32_t* block_table, int max_pages, int num_pages,
                          const int8_t* k8p, const int8_t* v8p, const int32_t* ek, const int32_t* ev,
                          const int32_t* ev0, int max_blocks, int split_blocks, int sink, void* out, int out_dtype,
                          const int64_t* os, void* stream);

/* ------------------------------------------------------------------------- self-test */

/* Test support, no counterpart in the reference: the failure path of the bounded waits.  Runs
 * lssab8_prefill_lattice (sink off, float32 out) with the TMA producer withholding key
 * block `withhold_block` of its first work item -- the pipeline barrier expects the block's bytes,
 * which never arrive -- and every wait limited to wait_us microseconds (1 .. 2,000,000) instead of
 * the usual ~2 s.  The kernel gives up, sets LSSAB8_DEV_TIMEOUT in the device error word, releases
 * its tensor memory and returns; the call returns LSSAB8_OK if the launch succeeded.  The next
 * call on the same context runs normally. */
int lssab8_selftest_timeout(const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
                            const int8_t* v8, const int32_t* ev, int B, int H, int KVH, int T, int dh,
                            int withhold_block, int wait_us, void* out, const int64_t* os, void* stream);

/* Test support, no counterpart in the reference: out[i] = the prefill epilogue's division of
 * y[i] by l[i] (l[i] != 0), i.e. the correctly rounded binary32 quotient the contract's
 * fl(O / l) names (reference/lssab8_golden.py:333).  Device pointers, n elements. */
int lssab8_selftest_div(const float* y, const float* l, long long n, float* out, void* stream);

/* Test support, no counterpart in the reference: the prefill fold's running-maximum rescale of
 * the pair x[2i], x[2i + 1] by D[i] (the contract's exponent-field subtraction with flush to +0,
 * reference/lssab8_golden.py:293-301; D <= 0 is the identity), followed by the fold's add of a
 * zero term.  Device pointers: x and out hold 2 * npairs floats, D npairs ints. */
int lssab8_selftest_rescale(const float* x, const int32_t* D, long long npairs, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LSSAB8_H */
