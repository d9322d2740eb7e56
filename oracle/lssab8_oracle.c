/*
 * LSSA-B8 / B9.1 CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's numpy golden, used as the checker for the CUDA
 * product path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library; the product path in lockstep_b200/ never does.
 *
 * Parity status: PINNED.  tests/golden/ holds digests and vectors produced by running the
 * reference itself (reference/lssab8_golden.py, reference/lssab8_torch.py,
 * reference/lssab9_golden.py, reference/lssab9_torch.py) on the reference selftest fixtures
 * and on the BASELINE configs; tests/test_oracle.py checks this file against them.
 *
 * Every function cites the reference lines it restates (paths relative to the reference
 * project root).  Arithmetic is exact integer work plus a fixed sequence of IEEE binary32
 * round-to-nearest-even operations; the library is compiled with -ffp-contract=off and
 * without -ffast-math so the compiler cannot change a single rounding.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#define OR_BHI 26                  /* reference/lssab8_golden.py:54            */
#define OR_KB 128                  /* reference/lssab8_golden.py:55            */
#define OR_SEG 32                  /* reference/lssab8_golden.py:56            */
#define OR_SWIN 32                 /* reference/lssab8_golden.py:69            */
#define OR_WLOC 9                  /* reference/lssab8_golden.py:70            */
#define OR_NIDX 7                  /* reference/lssab8_golden.py:71            */
#define OR_TOP 255                 /* reference/lssab8_golden.py:72            */
#define OR_TABLEN (17 << OR_NIDX)  /* reference/lssab8_golden.py:73 (KTAB_DOUB) */

/* error bits reported by the oracle (mirror the reference's asserts) */
#define OR_ERR_EV_RANGE 1          /* reference/lssab9_torch.py:158, lssab8_torch.py:152 */

static uint8_t g_t2[OR_TABLEN];
static int g_t2_ready = 0;

/* T2[k] = RN_half_up(255 * 2^(-k/128)) for k < 9*128, 0 beyond (reference/lssab8_golden.py:90-103).
 * Evaluated here in 80-bit long double; tests/test_oracle.py pins the result to the
 * contract digest sha256(csv) = 7a42a785...92fbb, so no precision argument is relied upon. */
static void or_build_t2(void) {
    if (g_t2_ready) return;
    for (int k = 0; k < OR_TABLEN; ++k) {
        if (k < (OR_WLOC << OR_NIDX)) {
            long double x = (long double)OR_TOP * exp2l(-(long double)k / (long double)(1 << OR_NIDX));
            g_t2[k] = (uint8_t)floorl(x + 0.5L);      /* half-up: all arguments are positive */
        } else {
            g_t2[k] = 0;
        }
    }
    g_t2_ready = 1;
}

int or_t2_table(uint8_t* out, int n) {
    or_build_t2();
    if (n < OR_TABLEN) return -1;
    memcpy(out, g_t2, OR_TABLEN);
    return OR_TABLEN;
}

/* ---------------------------------------------------------------- PREP (P1, P2, P3) */

/* The clip-safe pow2 exponent rule of contract_common.quant_pow2
 * (reference/contract_common.py:80-90; golden reference/lssab_golden.py:142-155; the B9
 * form with a 48 upper clamp reference/lssab9_golden.py:22-34):
 *   e = 7 - E (frexp), m == 0 -> 0, e -= 1 if m*2^e > 127, clamp [-32, hi]. */
static int or_exp_rule(float m, int hi) {
    if (m == 0.0f) return 0;
    int E;
    (void)frexpf(m, &E);
    int e = 7 - E;
    if (e <= 127) {                       /* m*2^e is exact in double for every such e */
        if (ldexp((double)m, e) > 127.0) e -= 1;
    } else {
        e -= 1;                           /* scale is inf in binary32: over is true */
    }
    if (e < -32) e = -32;
    if (e > hi) e = hi;
    return e;
}

static int8_t or_q8(float x, float sc) {
    float y = rintf(x * sc);              /* rint = round half to even */
    if (y > 127.0f) y = 127.0f;
    if (y < -127.0f) y = -127.0f;
    return (int8_t)y;
}

/* P1: per-row quantiser (reference/t10_attn.py:40-48, golden reference/lssab_golden.py:228-229).
 * x [nrows, dh] f32 -> q8 [nrows, dh], e [nrows]. */
void or_quant_rows(const float* x, int64_t nrows, int dh, int8_t* q8, int32_t* e) {
    for (int64_t r = 0; r < nrows; ++r) {
        const float* xr = x + r * dh;
        float m = 0.0f;
        for (int c = 0; c < dh; ++c) { float a = fabsf(xr[c]); if (a > m) m = a; }
        int ee = or_exp_rule(m, 40);
        float sc = ldexpf(1.0f, ee);
        for (int c = 0; c < dh; ++c) q8[r * dh + c] = or_q8(xr[c], sc);
        e[r] = ee;
    }
}

/* Quantise rows [r0, r1) of one [T, dh] tensor on ONE exponent (amax over the rows and all
 * channels).  reference/lssab_torch.py:62-85 (quant_pow2_blocks) and
 * reference/lssab9_torch.py:46-65 (quant_pow2_blocks_bits, 7 bits). */
static int or_quant_range(const float* x, int r0, int r1, int dh, int hi, int8_t* x8) {
    float m = 0.0f;
    for (int64_t i = (int64_t)r0 * dh; i < (int64_t)r1 * dh; ++i) { float a = fabsf(x[i]); if (a > m) m = a; }
    int ee = or_exp_rule(m, hi);
    float sc = ldexpf(1.0f, ee);
    for (int64_t i = (int64_t)r0 * dh; i < (int64_t)r1 * dh; ++i) x8[i] = or_q8(x[i], sc);
    return ee;
}

/* P2/P3: per-128-key-block K or V lattice for one kv head.  x [T, dh] -> x8 [T, dh], e [nblk].
 * mode 0: B8 (clamp [-32, 40]; reference/lssab_torch.py:62-85);
 * mode 1: B9 value grid (clamp [-32, 48], assert e in [-32, 40]; reference/lssab9_torch.py:123,158);
 * mode 2: B9.1 sink_alone value grid: key 0 alone -> *e0, keys 1..min(KB,T)-1 are block 0
 *         (reference/lssab9_torch.py:124-132, golden reference/lssab9_golden.py:51-58).
 * Returns an OR_ERR_* mask. */
int or_quant_blocks(const float* x, int T, int dh, int mode, int8_t* x8, int32_t* e, int32_t* e0) {
    int nblk = (T + OR_KB - 1) / OR_KB;
    int err = 0;
    int hi = (mode == 0) ? 40 : 48;
    for (int b = 0; b < nblk; ++b) {
        int lo = b * OR_KB, hi_r = (b + 1) * OR_KB < T ? (b + 1) * OR_KB : T;
        e[b] = or_quant_range(x, lo, hi_r, dh, hi, x8);
    }
    if (mode == 2 && T > 1) {
        int hi_r = OR_KB < T ? OR_KB : T;
        *e0 = or_quant_range(x, 0, 1, dh, 48, x8);
        e[0] = or_quant_range(x, 1, hi_r, dh, 48, x8);
    } else if (e0) {
        *e0 = 0;
    }
    if (mode != 0) {
        for (int b = 0; b < nblk; ++b) if (e[b] < -32 || e[b] > 40) err |= OR_ERR_EV_RANGE;
    }
    return err;
}

/* ------------------------------------------------------------------- fold helpers */


/* base = round(2^26 / (sqrt(dh) * ln 2)) with Python's round-half-even on the double
 * (reference/lssab_golden.py:161, reference/contract_common.py:94). */
int64_t or_gbase(int dh) {
    double x = ldexp(1.0, OR_BHI) / (sqrt((double)dh) * log(2.0));
    return (int64_t)nearbyint(x);
}

/* G = g_fold(dh, clamp(sh, -7, 23)) in [1, 2^30] (reference/lssab_golden.py:158-168). */
static int64_t or_gfold(int64_t base, int sh) {
    if (sh < -7) sh = -7;
    if (sh > 23) sh = 23;
    int64_t G;
    if (sh >= 0) G = (base + (sh > 0 ? ((int64_t)1 << (sh - 1)) : 0)) >> sh;
    else G = base << (-sh);
    if (G < 1) G = 1;
    if (G > ((int64_t)1 << 30)) G = (int64_t)1 << 30;
    return G;
}

/* The contract rescale: subtract D from the biased exponent field, flush to +0.0 when the
 * input is zero/subnormal or the result's biased exponent would be < 1
 * (reference/lssab8_golden.py:150-168). */
static float or_rescale(float x, int64_t D) {
    uint32_t u;
    memcpy(&u, &x, 4);
    int64_t e = (u >> 23) & 0xFF;
    int64_t ne = e - D;
    if (e >= 1 && ne >= 1) {
        u = (u & 0x807FFFFFu) | ((uint32_t)ne << 23);
        float y;
        memcpy(&y, &u, 4);
        return y;
    }
    return 0.0f;
}

int64_t or_floor_shift(int64_t x, int s) { return x >> s; }   /* arithmetic: floor */

/* ------------------------------------------------------------------------ the core
 *
 * lssab8_core (reference/lssab8_golden.py:200-338) with the B9.1 sink term of
 * lssab9_core (reference/lssab9_golden.py:189-224, groups eh0 then ehr on block 0).
 *
 *   q8 [H, T, dh], eq [H, T]              (row quantiser output)
 *   k8, v8 [KVH, T, dh], ek, ev [KVH, nblk] (block lattice; NOTE: kv-head major, the
 *                                           golden's [nblk, KVH] transposed)
 *   ev0 [KVH] or NULL                      (B9.1 sink exponent; NULL = sink off)
 *   d8 [KVH, T] or NULL                    (B9.3 per-key shift d_j of the PV weight,
 *                                           reference/lssab9_golden.py:37-41, 179-186)
 *   rows: the query rows to evaluate (NULL = all T rows); the key set of row i is
 *         { j : j <= i } when causal, { j : j < T } otherwise, further restricted to
 *         [key_lo, key_hi) (the split-KV segment restriction of lssab8_row_segments,
 *         reference/lssab8_golden.py:367-377) and to { j : kvalid[j] != 0 } when kvalid is
 *         not NULL (the golden's key_valid mask, reference/lssab8_golden.py:241-247).
 *   out [H, T, dh] f32 receives fl(O_row / l_row) (0 when l_row == 0) for evaluated rows.
 *   dbg_O [H, T, dh], dbg_l [H, T], dbg_nb [H, T] (optional): the row state before the
 *         division (NB_row stored as NB / 2^26; 0 when no block was visible).
 *   qrow >= 0: decode form -- q8 [H, 1, dh] and eq [H, 1] are the single query row that sits
 *         at position qrow; out/dbg are [H, 1, ...].  Identical to evaluating rows=[qrow] of
 *         the full problem (reference/lssab8_golden.py:207-209: rows are independent).
 */
typedef struct {
    int H, KVH, T, dh;
    const int8_t* q8; const int32_t* eq;
    const int8_t* k8; const int32_t* ek;
    const int8_t* v8; const int32_t* ev;
    const int32_t* ev0;
    const int8_t* d8;    /* B9.3 per-key weight shift [KVH, T] (NULL: none) */
    int causal;
    int key_lo, key_hi;
    int qrow;            /* >= 0: q8/eq hold ONE row per head, standing for query row qrow */
    const uint8_t* kvalid;   /* [T] key mask (NULL: every key) */
} or_problem;

static void or_row(const or_problem* P, int h, int i, float* out_row, float* dO, float* dl, int64_t* dnb,
                   int32_t* S, int32_t* eh, int32_t* A0, int32_t* A1, float* Oseg, float* Orow) {
    const int T = P->T, dh = P->dh, KVH = P->KVH;
    const int grp = P->H / KVH;
    const int g = h / grp;
    const int nblk = (T + OR_KB - 1) / OR_KB;
    const int nseg = (nblk + OR_SEG - 1) / OR_SEG;
    const int64_t base = or_gbase(dh);
    const int64_t qi = (P->qrow >= 0) ? (int64_t)h : ((int64_t)h * T + i);
    const int8_t* qrow = P->q8 + qi * dh;
    const int eqi = P->eq[qi];
    const int8_t* kg = P->k8 + (int64_t)g * T * dh;
    const int8_t* vg = P->v8 + (int64_t)g * T * dh;
    const int64_t win_d = (int64_t)OR_WLOC << OR_BHI;     /* masked keys -> zero weight */
    const int idx_sh = OR_BHI - OR_NIDX;

    for (int c = 0; c < dh; ++c) Orow[c] = 0.0f;
    float lrow = 0.0f;
    int have_row = 0;
    int64_t nb_row = 0;

    for (int sg = 0; sg < nseg; ++sg) {
        int b0 = sg * OR_SEG, b1 = (sg + 1) * OR_SEG < nblk ? (sg + 1) * OR_SEG : nblk;
        for (int c = 0; c < dh; ++c) Oseg[c] = 0.0f;
        float lseg = 0.0f;
        int have_seg = 0;
        int64_t nb_run = 0;
        for (int b = b0; b < b1; ++b) {
            int lo = b * OR_KB, hi = (b + 1) * OR_KB < T ? (b + 1) * OR_KB : T;
            int n = hi - lo;
            int any = 0;
            int32_t mS = INT32_MIN;
            for (int t = 0; t < n; ++t) {
                int j = lo + t;
                int vis = (j >= P->key_lo && j < P->key_hi) && (!P->causal || j <= i) &&
                          (!P->kvalid || P->kvalid[j]);
                const int8_t* kr = kg + (int64_t)j * dh;
                int32_t s = 0;
                for (int c = 0; c < dh; ++c) s += (int32_t)qrow[c] * (int32_t)kr[c];
                S[t] = vis ? s : INT32_MIN;
                if (vis) { any = 1; if (s > mS) mS = s; }
            }
            if (!any) continue;
            int64_t G = or_gfold(base, eqi + P->ek[(int64_t)g * nblk + b]);
            int64_t SGm = (int64_t)mS * G;
            int64_t NB = -((-SGm) >> OR_BHI) << OR_BHI;       /* least multiple of 2^26 >= SGm */
            if (!have_seg) { nb_run = NB; have_seg = 1; }
            int64_t D = (NB - nb_run) >> OR_BHI;
            int64_t s;
            if (D > 0) {
                for (int c = 0; c < dh; ++c) Oseg[c] = or_rescale(Oseg[c], D);
                lseg = or_rescale(lseg, D);
                nb_run = NB; s = 0;
            } else {
                s = -D;
                if (s > OR_SWIN) continue;                     /* the exact skip */
            }
            /* the chain (exact integers) reference/lssab8_golden.py:281-293 */
            int64_t lb = 0;
            for (int t = 0; t < n; ++t) {
                int64_t d = (S[t] == INT32_MIN) ? win_d : NB - (int64_t)S[t] * G;
                int64_t k = d >> idx_sh;
                if (k > OR_TABLEN - 1) k = OR_TABLEN - 1;
                eh[t] = g_t2[k];
                lb += eh[t];
            }
            /* block partials reference/lssab8_golden.py:295-301; B9.1 groups
             * reference/lssab9_golden.py:189-196 (block 0 only, key 0 first) */
            int sink = (P->ev0 != NULL) && (b == 0) && (lo == 0) && (T > 1);
            for (int c = 0; c < dh; ++c) { A0[c] = 0; A1[c] = 0; }
            for (int t = 0; t < n; ++t) {
                /* B9.3: the PV weight is eh >> d_j, l_b keeps the unshifted weight
                 * (reference/lssab9_golden.py:179-186, default truncating shift) */
                const int32_t w = P->d8 ? (eh[t] >> P->d8[(int64_t)g * T + lo + t]) : eh[t];
                if (w == 0) continue;
                const int8_t* vr = vg + (int64_t)(lo + t) * dh;
                int32_t* A = (sink && t == 0) ? A0 : A1;
                for (int c = 0; c < dh; ++c) A[c] += w * (int32_t)vr[c];
            }
            int nz = (lb != 0);
            for (int c = 0; c < dh && !nz; ++c) nz = (A0[c] != 0) || (A1[c] != 0);
            if (!nz) continue;
            /* the fold, fp32 RNE, committed order reference/lssab8_golden.py:304-313 */
            int evb = P->ev[(int64_t)g * nblk + b];
            if (sink) {
                float sc0 = ldexpf(1.0f, (int)(-(s + P->ev0[g])));
                for (int c = 0; c < dh; ++c) { float t0 = (float)A0[c] * sc0; Oseg[c] = Oseg[c] + t0; }
            }
            float scO = ldexpf(1.0f, (int)(-(s + evb)));
            float scl = ldexpf(1.0f, (int)(-s));
            for (int c = 0; c < dh; ++c) { float t1 = (float)A1[c] * scO; Oseg[c] = Oseg[c] + t1; }
            { float tl = (float)lb * scl; lseg = lseg + tl; }
        }
        if (!have_seg) continue;
        /* segment -> row, the same three rules (reference/lssab8_golden.py:317-331) */
        if (!have_row) { nb_row = nb_run; have_row = 1; }
        int64_t D = (nb_run - nb_row) >> OR_BHI;
        int64_t s;
        if (D > 0) {
            for (int c = 0; c < dh; ++c) Orow[c] = or_rescale(Orow[c], D);
            lrow = or_rescale(lrow, D);
            nb_row = nb_run; s = 0;
        } else {
            s = -D;
            if (s > OR_SWIN) continue;
        }
        for (int c = 0; c < dh; ++c) Orow[c] = Orow[c] + or_rescale(Oseg[c], s);
        lrow = lrow + or_rescale(lseg, s);
    }
    if (dO) for (int c = 0; c < dh; ++c) dO[c] = Orow[c];
    if (dl) *dl = lrow;
    if (dnb) *dnb = have_row ? (nb_row >> OR_BHI) : 0;
    /* epilogue: one correctly rounded division, l == 0 -> 0 (reference/lssab8_golden.py:334-335) */
    if (lrow != 0.0f) { for (int c = 0; c < dh; ++c) out_row[c] = Orow[c] / lrow; }
    else { for (int c = 0; c < dh; ++c) out_row[c] = 0.0f; }
}

/* Evaluate rows (all rows when rows == NULL) of every head.  Threads over (head, row). */
int or_core(int H, int KVH, int T, int dh,
            const int8_t* q8, const int32_t* eq, const int8_t* k8, const int32_t* ek,
            const int8_t* v8, const int32_t* ev, const int32_t* ev0, const int8_t* d8,
            int causal, int key_lo, int key_hi,
            const int32_t* rows, int nrows,
            float* out, float* dbg_O, float* dbg_l, int64_t* dbg_nb, int nthreads, int qrow,
            const uint8_t* kvalid) {
    or_build_t2();
    if (H <= 0 || KVH <= 0 || H % KVH != 0 || T <= 0 || dh <= 0 || dh > 256) return -1;
    if (qrow >= T) return -1;
    if (rows && qrow < 0) {
        for (int r = 0; r < nrows; ++r) if (rows[r] < 0 || rows[r] >= T) return -1;
    }
    or_problem P = { H, KVH, T, dh, q8, eq, k8, ek, v8, ev, ev0, d8, causal, key_lo, key_hi, qrow, kvalid };
    int nr = (qrow >= 0) ? 1 : (rows ? nrows : T);
    int64_t total = (int64_t)H * nr;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
    {
        int32_t* S = (int32_t*)malloc(sizeof(int32_t) * OR_KB * 2);
        int32_t* eh = S + OR_KB;
        int32_t* A0 = (int32_t*)malloc(sizeof(int32_t) * dh * 2);
        int32_t* A1 = A0 + dh;
        float* Oseg = (float*)malloc(sizeof(float) * dh * 2);
        float* Orow = Oseg + dh;
#pragma omp for schedule(dynamic, 4)
        for (int64_t w = 0; w < total; ++w) {
            int h = (int)(w / nr);
            int i = (qrow >= 0) ? qrow : (rows ? rows[w % nr] : (int)(w % nr));
            /* single-row mode writes out/dbg as [H, 1, ...] */
            int64_t o = (qrow >= 0) ? (int64_t)h : ((int64_t)h * T + i);
            or_row(&P, h, i, out + o * dh, dbg_O ? dbg_O + o * dh : NULL, dbg_l ? dbg_l + o : NULL,
                   dbg_nb ? dbg_nb + o : NULL, S, eh, A0, A1, Oseg, Orow);
        }
        free(S); free(A0); free(Oseg);
    }
    return 0;
}
