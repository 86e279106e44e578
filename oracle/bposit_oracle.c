/*
 * bposit_oracle.c -- CPU restatement of the open-bposit W8A8 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle that the CUDA library
 * (open-bposit_b200/csrc) is compared against.  Only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference arm of bench.py may load
 * it; no product code path calls it, and the product fails loudly when its own
 * CUDA library is missing instead of falling back to this file.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function here against
 * golden vectors produced by running the reference itself (tests/golden/, made
 * by tests/golden/make_golden.py): the reference's encoder vectors
 * (reference/gen_encoder_vectors.py), the exhaustive bp8 product vectors
 * (reference/gen_bp8_exhaustive.py), the bp8 RTL dots (reference/gen_rtl_vectors.py),
 * the bposit_fast self-test dots (reference/bposit_fast.py:179-197), all bp8 /
 * bp16 codes, and quantize_bp8 / encode_bposit16 outputs on seeded inputs.
 *
 * The algorithms deliberately follow the reference's own formulation (bit
 * loops, a sorted grid with searchsorted, shift-class quire sums), not the
 * table/bit-twiddling formulation of the device kernels, so that the two are
 * independent statements of the same semantics.
 *
 * Citations are relative to the reference project root.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>
#include <math.h>
#include <pthread.h>

#define QFRAC 96   /* QUIRE_FRAC_BITS, reference/bposit_ref.py:541 */

/* ------------------------------------------------------------------------ */
/* Generic posit field decode: reference/bposit_ref.py:162-193 (bp8),        */
/* :306-355 (bp16), :43-74 (bp32).  Returns 0 for zero, -1 for NaR, else 1.  */
/* The value is  (-1)^sign * useed^k * 2^e * (1 + fbits/2^fw)                */
/* = sign * mant * 2^exp with mant = 2^fw + fbits, exp = k*2^es + e - fw.    */
/* ------------------------------------------------------------------------ */
static int decode_field(uint32_t p, int nbits, int es, int *sign_out, int64_t *mant, int *exp)
{
    uint32_t mask = (nbits == 32) ? 0xFFFFFFFFu : ((1u << nbits) - 1u);
    p &= mask;
    uint32_t nar = 1u << (nbits - 1);
    if (p == 0) { *mant = 0; *exp = 0; *sign_out = 0; return 0; }
    if (p == nar) { *mant = 0; *exp = 0; *sign_out = 0; return -1; }
    int sign = (p >> (nbits - 1)) & 1;
    uint32_t rest_mask = nar - 1u;
    uint32_t rest = p & rest_mask;
    if (sign) rest = ((~rest) + 1u) & rest_mask;
    int top = nbits - 2;
    int leading = (rest >> top) & 1;
    int rs = 0;
    while (rs < nbits - 1 && (int)((rest >> (top - rs)) & 1) == leading) rs++;
    int k, e = 0, fw = 0;
    uint32_t fbits = 0;
    if (rs == nbits - 1) {
        k = leading ? (nbits - 2) : -(nbits - 1);
    } else {
        k = leading ? (rs - 1) : -rs;
        int remaining = (nbits - 1) - (rs + 1);
        uint32_t rest2 = remaining > 0 ? (rest & ((1u << remaining) - 1u)) : 0u;
        int ew = remaining < es ? remaining : es;
        if (ew > 0) {
            e = (int)((rest2 >> (remaining - ew)) & ((1u << ew) - 1u));
            e <<= (es - ew);
        }
        remaining -= ew;
        fw = remaining;
        fbits = fw > 0 ? (rest2 & ((1u << fw) - 1u)) : 0u;
    }
    *sign_out = sign;
    int64_t m = ((int64_t)1 << fw) + (int64_t)fbits;
    *mant = sign ? -m : m;
    *exp = k * (1 << es) + e - fw;
    return 1;
}

/* code -> (signed mantissa, exponent); zero and NaR -> mant 0, like code_value
 * (reference/bposit_ref.py:1022-1025) and the bp8 ROM of gen_rtl_vectors.py:289-298. */
static int es_of(int fmt_bits)
{
    return fmt_bits <= 5 ? 1 : (fmt_bits == 8 ? 2 : 3);   /* bp4/aip5: 1, bp8: 2, bp16/bp32: 3 */
}

void orc_decode_me(int fmt_bits, uint32_t code, int64_t *mant, int *exp)
{
    int s;
    int es = es_of(fmt_bits);
    int r = decode_field(code, fmt_bits, es, &s, mant, exp);
    if (r <= 0) { *mant = 0; *exp = 0; }
}

/* code -> double value (exact for bp8 / bp16); NaR -> NaN here, zero -> 0. */
static double decode_double(int fmt_bits, uint32_t code)
{
    int s; int64_t m; int e;
    int es = fmt_bits == 8 ? 2 : 3;
    int r = decode_field(code, fmt_bits, es, &s, &m, &e);
    if (r == 0) return 0.0;
    if (r < 0) return NAN;
    return ldexp((double)m, e);
}

/* Decode codes to fp32 values (the bp8 and bp16 values are exact in fp32).
 * NaR decodes to 0, matching code_value. */
void orc_decode_f32(int fmt_bits, const void *codes, size_t n, float *out)
{
    for (size_t i = 0; i < n; i++) {
        uint32_t c = fmt_bits == 8 ? ((const uint8_t *)codes)[i] : ((const uint16_t *)codes)[i];
        int64_t m; int e;
        orc_decode_me(fmt_bits, c, &m, &e);
        out[i] = (float)ldexp((double)m, e);
    }
}

/* ------------------------------------------------------------------------ */
/* bp8 quantize: reference/bposit_fast.py:49-99 (_grid, _mids, quantize_bp8) */
/* ------------------------------------------------------------------------ */
static double g_grid[128], g_mids[127];
static int g_grid_ready = 0;
static pthread_once_t g_grid_once = PTHREAD_ONCE_INIT;

static int cmp_double(const void *a, const void *b)
{
    double x = *(const double *)a, y = *(const double *)b;
    return (x > y) - (x < y);
}

static void build_grid(void)
{
    /* sorted(set(|code_value(c)| for c in 0..255)) -- bposit_fast.py:53 */
    double mags[256];
    int n = 0;
    for (int c = 0; c < 256; c++) {
        int64_t m; int e;
        orc_decode_me(8, (uint32_t)c, &m, &e);
        double v = fabs(ldexp((double)m, e));
        int seen = 0;
        for (int j = 0; j < n; j++) if (mags[j] == v) { seen = 1; break; }
        if (!seen) mags[n++] = v;
    }
    qsort(mags, (size_t)n, sizeof(double), cmp_double);
    /* n == 128 */
    for (int i = 0; i < 128; i++) g_grid[i] = mags[i];
    for (int i = 0; i < 127; i++) g_mids[i] = (g_grid[i] + g_grid[i + 1]) / 2.0; /* :65 */
    g_grid_ready = 1;
}

static void ensure_grid(void) { pthread_once(&g_grid_once, build_grid); }

void orc_bp8_grid(double *grid128, double *mids127)
{
    ensure_grid();
    memcpy(grid128, g_grid, sizeof g_grid);
    memcpy(mids127, g_mids, sizeof g_mids);
}

/* numpy searchsorted(arr, a, side="left"): first i with arr[i] >= a. */
static int ss_left(const double *arr, int n, double a)
{
    int lo = 0, hi = n;
    while (lo < hi) { int mid = (lo + hi) / 2; if (arr[mid] < a) lo = mid + 1; else hi = mid; }
    return lo;
}
/* side="right": first i with arr[i] > a. */
static int ss_right(const double *arr, int n, double a)
{
    int lo = 0, hi = n;
    while (lo < hi) { int mid = (lo + hi) / 2; if (arr[mid] <= a) lo = mid + 1; else hi = mid; }
    return lo;
}

/* One element of quantize_bp8 (reference/bposit_fast.py:89-99), returning the
 * bp8 code of the quantized value (value->code as examples/w8a8_rounding_demo.py:31:
 * +g[i] -> i, -g[i] -> (-i) & 0xFF, +-0 -> 0).  NaN has no code in the reference
 * (its quantized value is NaN); it is mapped to NaR 0x80. */
static uint8_t quantize_one(double x, int nearest)
{
    if (isnan(x)) return 0x80;
    double a = fabs(x);
    int idx;
    if (nearest) idx = ss_left(g_mids, 127, a);
    else idx = ss_right(g_grid, 128, a) - 1;
    if (idx < 0) idx = 0;
    if (idx > 127) idx = 127;
    if (a > 0 && a < g_grid[1]) idx = 1;           /* tiny override, :97-98 */
    if (idx == 0) return 0;
    return (uint8_t)(x < 0 ? ((256 - idx) & 0xFF) : idx);
}

/* float64 entry (the reference's own input dtype, bposit_fast.py:90) */
void orc_quantize_bp8_f64(const double *x, size_t n, int nearest, uint8_t *codes)
{
    ensure_grid();
    for (size_t i = 0; i < n; i++) codes[i] = quantize_one(x[i], nearest);
}

void orc_quantize_bp8(const float *x, size_t n, int nearest, uint8_t *codes, float *values)
{
    ensure_grid();
    for (size_t i = 0; i < n; i++) {
        uint8_t c = quantize_one((double)x[i], nearest);
        if (codes) codes[i] = c;
        if (values) {
            if (isnan(x[i])) values[i] = NAN;
            else values[i] = (float)decode_double(8, c);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* bp16 encode, exact-rational entry: _encode_unsigned(value, mode) and      */
/* encode_bposit16 (reference/bposit_ref.py:382-507) on value = Fraction(x). */
/* A float input is exact as a double, and every step of the bit loop        */
/* (halving/doubling, f*=2, f-=1) stays exact in double precision.          */
/* mode: 0 = "truncate", 1 = "rtne".                                        */
/* ------------------------------------------------------------------------ */
static uint32_t encode_unsigned16(double value, int rtne)
{
    if (value == 0) return 0;
    int total_e = 0;
    double v = value;
    if (v >= 1) { while (v >= 2) { v /= 2; total_e++; } }
    else { while (v < 1) { v *= 2; total_e--; } }
    if (total_e > 112) return 0x7FFF;
    if (total_e < -112) return 0x0001;
    int k = total_e >> 3;             /* floor division, Python semantics */
    int e = total_e & 7;
    double f = v - 1;
    int bits[40]; int nb = 0;
    if (k >= 0) { for (int i = 0; i < k + 1; i++) bits[nb++] = 1; bits[nb++] = 0; }
    else { for (int i = 0; i < -k; i++) bits[nb++] = 0; bits[nb++] = 1; }
    int round_up = 0;
    if (nb >= 15) {
        nb = 15;
    } else {
        for (int i = 2; i >= 0; i--) {
            bits[nb++] = (e >> i) & 1;
            if (nb == 15) break;
        }
        while (nb < 16) {
            f *= 2;
            if (f >= 1) { bits[nb++] = 1; f -= 1; } else bits[nb++] = 0;
        }
        int round_bit = nb > 15 ? bits[15] : 0;
        nb = 15;
        if (rtne) {
            int sticky = f > 0;
            int lsb_odd = bits[14] == 1;
            round_up = round_bit == 1 && (sticky || lsb_odd);
        }
    }
    uint32_t out = 0;
    for (int i = 0; i < nb; i++) out = (out << 1) | (uint32_t)bits[i];
    out <<= (15 - nb);
    out &= 0x7FFF;
    if (rtne && round_up && out < 0x7FFF) out += 1;
    return out;
}

/* fp32 -> bp16.  NaN -> NaR 0x8000 and +-inf -> +-maxpos are extensions (the
 * reference raises on non-finite input: Fraction(nan)/Fraction(inf)). */
uint16_t orc_encode_bp16_one(float x, int rtne)
{
    if (isnan(x)) return 0x8000;
    double d = (double)x;
    if (d == 0) return 0;
    int sign = d < 0;
    double a = fabs(d);
    uint32_t field;
    if (isinf(a)) field = 0x7FFF;
    else field = encode_unsigned16(a, rtne);
    if (sign) field = ((~field) + 1u) & 0x7FFF;
    return (uint16_t)(((uint32_t)sign << 15 | field) & 0xFFFF);
}

void orc_encode_bp16(const float *x, size_t n, int rtne, uint16_t *codes)
{
    for (size_t i = 0; i < n; i++) codes[i] = orc_encode_bp16_one(x[i], rtne);
}

/* ------------------------------------------------------------------------ */
/* Quire: two's complement integer with QFRAC fraction bits, 16 x 32-bit     */
/* limbs (512 bits), little-endian.  The reference uses unbounded Python     */
/* ints; 512 bits hold every bp16 quire (|q| < 2^352 for K < 2^32).          */
/* ------------------------------------------------------------------------ */
#define QL 16
typedef struct { uint32_t w[QL]; } quire_t;

static void q_zero(quire_t *q) { memset(q, 0, sizeof *q); }

/* q += v * 2^sh, v signed 64-bit, sh >= 0 */
static void q_add_shifted(quire_t *q, int64_t v, int sh)
{
    if (v == 0) return;
    /* build the 512-bit two's complement of v<<sh and add */
    uint32_t t[QL];
    uint64_t uv = (uint64_t)v;
    uint32_t fill = v < 0 ? 0xFFFFFFFFu : 0u;
    for (int i = 0; i < QL; i++) t[i] = fill;
    /* place 64-bit v at bit offset sh, sign-extended */
    int limb = sh / 32, bit = sh % 32;
    /* the 96-bit value (sign-extended v) << bit, spread over 3 limbs */
    uint32_t lo = (uint32_t)uv, hi = (uint32_t)(uv >> 32);
    uint32_t x0, x1, x2;
    if (bit == 0) { x0 = lo; x1 = hi; x2 = fill; }
    else {
        x0 = lo << bit;
        x1 = (hi << bit) | (lo >> (32 - bit));
        x2 = (fill << bit) | (hi >> (32 - bit));
    }
    for (int i = 0; i < limb && i < QL; i++) t[i] = 0;
    if (limb < QL) t[limb] = x0;
    if (limb + 1 < QL) t[limb + 1] = x1;
    if (limb + 2 < QL) t[limb + 2] = x2;
    uint64_t carry = 0;
    for (int i = 0; i < QL; i++) {
        uint64_t s = (uint64_t)q->w[i] + t[i] + carry;
        q->w[i] = (uint32_t)s;
        carry = s >> 32;
    }
}

static int q_is_neg(const quire_t *q) { return (q->w[QL - 1] >> 31) & 1; }

static void q_neg(quire_t *q)
{
    uint64_t carry = 1;
    for (int i = 0; i < QL; i++) {
        uint64_t s = (uint64_t)(uint32_t)(~q->w[i]) + carry;
        q->w[i] = (uint32_t)s;
        carry = s >> 32;
    }
}

static int q_bit(const quire_t *q, int i) { return (q->w[i / 32] >> (i % 32)) & 1; }

/* quire256_to_bposit32 -> encode_bposit32 -> _encode_unsigned_32
 * (reference/bposit_ref.py:703-722, 138-150, 97-135): the exact value
 * q / 2^96, truncated to a bposit32 (eS=3) bit string. */
static uint32_t q_to_bp32(const quire_t *qin)
{
    quire_t q = *qin;
    int nz = 0;
    for (int i = 0; i < QL; i++) nz |= q.w[i] != 0;
    if (!nz) return 0;
    int sign = q_is_neg(&q);
    if (sign) q_neg(&q);
    int msb = -1;
    for (int i = QL * 32 - 1; i >= 0; i--) if (q_bit(&q, i)) { msb = i; break; }
    int total_e = msb - QFRAC;       /* floor(log2(|q| / 2^96)) */
    uint32_t field;
    if (total_e > 240) field = 0x7FFFFFFF;
    else if (total_e < -240) field = 0x00000001;
    else {
        int k = total_e >> 3, e = total_e & 7;
        int bits[80]; int nb = 0;
        if (k >= 0) { for (int i = 0; i < k + 1; i++) bits[nb++] = 1; bits[nb++] = 0; }
        else { for (int i = 0; i < -k; i++) bits[nb++] = 0; bits[nb++] = 1; }
        if (nb >= 31) nb = 31;
        else {
            for (int i = 2; i >= 0; i--) { bits[nb++] = (e >> i) & 1; if (nb == 31) break; }
            /* fraction f = v - 1: the bits of |q| below its msb, MSB first */
            int pos = msb - 1;
            while (nb < 32) { bits[nb++] = pos >= 0 ? q_bit(&q, pos) : 0; pos--; }
            if (nb > 31) nb = 31;
        }
        uint32_t out = 0;
        for (int i = 0; i < nb; i++) out = (out << 1) | (uint32_t)bits[i];
        out <<= (31 - nb);
        field = out & 0x7FFFFFFF;
    }
    if (sign) field = ((~field) + 1u) & 0x7FFFFFFF;
    return ((uint32_t)sign << 31) | field;
}

/* Round a quire given as little-endian 32-bit limbs (two's complement,
 * nlimbs <= 16, sign-extended to 512 bits) to bposit32. */
uint32_t orc_quire_to_bp32(const uint32_t *limbs, int nlimbs)
{
    quire_t q;
    uint32_t fill = (limbs[nlimbs - 1] >> 31) ? 0xFFFFFFFFu : 0u;
    for (int i = 0; i < QL; i++) q.w[i] = i < nlimbs ? limbs[i] : fill;
    return q_to_bp32(&q);
}

void orc_quire_to_bp32_batch(const uint32_t *limbs, int nlimbs, size_t n, uint32_t *out)
{
    for (size_t i = 0; i < n; i++) out[i] = orc_quire_to_bp32(limbs + i * (size_t)nlimbs, nlimbs);
}

/* quire256_to_bposit16 (reference/bposit_ref.py:620-635): |q| / 2^96 through
 * encode_bposit16 in its default "truncate" mode, _encode_unsigned
 * (reference/bposit_ref.py:382-486): regime, up to three exponent bits
 * (MSB first), fraction bits, cut to the 15-bit field; total_e > 112 ->
 * maxpos 0x7FFF, total_e < -112 -> minpos 0x0001; negative values take the
 * two's complement of the field (reference/bposit_ref.py:503-507). */
static uint16_t q_to_bp16(const quire_t *qin)
{
    quire_t q = *qin;
    int nz = 0;
    for (int i = 0; i < QL; i++) nz |= q.w[i] != 0;
    if (!nz) return 0;
    int sign = q_is_neg(&q);
    if (sign) q_neg(&q);
    int msb = -1;
    for (int i = QL * 32 - 1; i >= 0; i--) if (q_bit(&q, i)) { msb = i; break; }
    int total_e = msb - QFRAC;
    uint32_t field;
    if (total_e > 112) field = 0x7FFF;
    else if (total_e < -112) field = 0x0001;
    else {
        int k = total_e >> 3, e = total_e & 7;
        int bits[40]; int nb = 0;
        if (k >= 0) { for (int i = 0; i < k + 1; i++) bits[nb++] = 1; bits[nb++] = 0; }
        else { for (int i = 0; i < -k; i++) bits[nb++] = 0; bits[nb++] = 1; }
        if (nb >= 15) nb = 15;
        else {
            for (int i = 2; i >= 0; i--) { bits[nb++] = (e >> i) & 1; if (nb == 15) break; }
            int pos = msb - 1;
            while (nb < 16) { bits[nb++] = pos >= 0 ? q_bit(&q, pos) : 0; pos--; }
            nb = 15;
        }
        uint32_t out = 0;
        for (int i = 0; i < nb; i++) out = (out << 1) | (uint32_t)bits[i];
        out <<= (15 - nb);
        field = out & 0x7FFF;
    }
    if (sign) field = ((~field) + 1u) & 0x7FFF;
    return (uint16_t)(((uint32_t)sign << 15) | field);
}

void orc_quire_to_bp16_batch(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out)
{
    for (size_t i = 0; i < n; i++) {
        const uint32_t *l = limbs + i * (size_t)nlimbs;
        quire_t q;
        uint32_t fill = (l[nlimbs - 1] >> 31) ? 0xFFFFFFFFu : 0u;
        for (int j = 0; j < QL; j++) q.w[j] = j < nlimbs ? l[j] : fill;
        out[i] = q_to_bp16(&q);
    }
}

/* Small rungs: _encode_unsigned_gen + _encode_gen (reference/bposit_ref.py:806-866)
 * in truncate mode for bposit4 (nbits 4, es 1, max_e 2) and AI-posit5
 * (nbits 5, es 1, max_e 4) on float64 input: |x| whose limit_denominator(10**8)
 * is 0 gives code 0; floor(log2|x|) > max_e -> maxpos field, < -max_e -> minpos;
 * else regime bits, es exponent bits, fraction bits cut to nbits-1 bits; the
 * sign takes the field's two's complement. */
static uint32_t small_encode_one(double x, int nbits, int es, int max_e)
{
    int F = nbits - 1;
    uint32_t fmask = (1u << F) - 1u;
    if (x != x) return 1u << F;
    int sign = x < 0;
    double a = fabs(x);
    /* limit_denominator(10**8) is 0 iff a < 1/(2*10^8); the largest double
     * below that rational is 0x1.5798ee2308c39p-28 */
    if (a <= 0x1.5798ee2308c39p-28) return 0;
    uint32_t field;
    if (isinf(a)) field = fmask;
    else {
        int te;
        double m = frexp(a, &te);   /* a = m 2^te, m in [0.5, 1) */
        te -= 1;                    /* floor(log2 a) */
        if (te > max_e) field = fmask;
        else if (te < -max_e) field = 1u;
        else {
            int k = te >= 0 ? te >> es : -((-te + (1 << es) - 1) >> es);   /* floor(te / 2^es) */
            int e = te - k * (1 << es);
            int bits[64]; int nb = 0;
            if (k >= 0) { for (int i = 0; i < k + 1; i++) bits[nb++] = 1; bits[nb++] = 0; }
            else { for (int i = 0; i < -k; i++) bits[nb++] = 0; bits[nb++] = 1; }
            if (nb >= F) nb = F;
            else {
                for (int i = es - 1; i >= 0; i--) { bits[nb++] = (e >> i) & 1; if (nb == F) break; }
                double f = 2.0 * m - 1.0;      /* fraction of a / 2^te in [0, 1), exact */
                while (nb < F + 1) { f *= 2.0; if (f >= 1.0) { bits[nb++] = 1; f -= 1.0; } else bits[nb++] = 0; }
                nb = F;
            }
            uint32_t out = 0;
            for (int i = 0; i < nb; i++) out = (out << 1) | (uint32_t)bits[i];
            out <<= (F - nb);
            field = out & fmask;
        }
    }
    if (sign) field = ((~field) + 1u) & fmask;
    return ((uint32_t)sign << F) | field;
}

void orc_quantize_small(int nbits, const double *x, size_t n, uint8_t *codes)
{
    int max_e = nbits == 4 ? 2 : 4;
    for (size_t i = 0; i < n; i++) codes[i] = (uint8_t)small_encode_one(x[i], nbits, 1, max_e);
}

/* Exact transcode to a wider format: the code of the same value (NaR -> NaR). */
void orc_transcode(int fmt_in, int fmt_out, const uint8_t *in, size_t n, void *out)
{
    int es_in = es_of(fmt_in), es_out = es_of(fmt_out);
    uint32_t lut[256];
    for (uint32_t c = 0; c < (1u << fmt_in); c++) {
        int s; int64_t m; int e;
        int r = decode_field(c, fmt_in, es_in, &s, &m, &e);
        uint32_t nar_out = 1u << (fmt_out - 1);
        if (r == 0) { lut[c] = 0; continue; }
        if (r < 0) { lut[c] = nar_out; continue; }
        double v = ldexp((double)m, e);
        lut[c] = nar_out;
        for (uint32_t d = 1; d < (1u << fmt_out); d++) {
            int s2; int64_t m2; int e2;
            if (decode_field(d, fmt_out, es_out, &s2, &m2, &e2) > 0 && ldexp((double)m2, e2) == v) { lut[c] = d; break; }
        }
    }
    for (size_t i = 0; i < n; i++) {
        uint32_t v = lut[in[i] & ((1u << fmt_in) - 1u)];
        if (fmt_out == 8) ((uint8_t *)out)[i] = (uint8_t)v;
        else ((uint16_t *)out)[i] = (uint16_t)v;
    }
}

/* ------------------------------------------------------------------------ */
/* Per-group power-of-two scale: s = ceil(log2(absmax / maxpos_bp8)) with    */
/* maxpos_bp8 = 2^24 (reference/bposit_ref.py:226-227), i.e.                 */
/* ceil_log2(absmax) - 24, computed exactly from frexp; absmax 0 -> 0.       */
/* ------------------------------------------------------------------------ */
static int ceil_log2_exact(double a)
{
    int e;
    double m = frexp(a, &e);     /* a = m * 2^e, m in [0.5, 1) */
    return m == 0.5 ? e - 1 : e;
}

void orc_group_scales(const float *x, int rows, int K, int group, int maxpos_log2, int32_t *s)
{
    int G = (K + group - 1) / group;
    for (int r = 0; r < rows; r++)
        for (int g = 0; g < G; g++) {
            double amax = 0;
            for (int k = g * group; k < K && k < (g + 1) * group; k++) {
                double a = fabs((double)x[(size_t)r * K + k]);
                if (a > amax) amax = a;
            }
            s[(size_t)r * G + g] = amax > 0 ? ceil_log2_exact(amax) - maxpos_log2 : 0;
        }
}

/* Quantize rows with per-group scales: code = quantize_bp8(x / 2^s, nearest). */
void orc_quantize_bp8_grouped(const float *x, int rows, int K, int group, const int32_t *s,
                              int nearest, uint8_t *codes)
{
    ensure_grid();
    int G = (K + group - 1) / group;
    for (int r = 0; r < rows; r++)
        for (int k = 0; k < K; k++) {
            double v = ldexp((double)x[(size_t)r * K + k], -s[(size_t)r * G + k / group]);
            codes[(size_t)r * K + k] = quantize_one(v, nearest);
        }
}

/* ------------------------------------------------------------------------ */
/* Exact quire GEMM: q[m][n] = sum_k trunc0(v(A[m,k]) * v(B[n,k]) *          */
/*                                          2^(sa[m,g] + sb[n,g]) * 2^96)    */
/* -- dot_at_precision's per-term rule (reference/bposit_ref.py:1028-1035)   */
/* with the optional group scale folded in as an exact power of two, and     */
/* bposit_fast's shift-class evaluation (reference/bposit_fast.py:102-128):  */
/* int64 sums per bit shift, one wide shift-add per class, per-term          */
/* truncation toward zero for negative shifts.                               */
/* ------------------------------------------------------------------------ */
typedef struct {
    int fmt_bits, M, N, K, group, G;
    const void *A, *B;
    const int32_t *sa, *sb;
    uint32_t *out_bp32;
    uint32_t *out_quire; int nlimbs;
    int row0, row1;
    const int64_t *mA; const int *eA; /* per-code tables */
} gemm_job;

#define SHIFT_MIN (-640)
#define SHIFT_MAX 640
#define NSHIFT (SHIFT_MAX - SHIFT_MIN + 1)

static void *gemm_worker(void *arg)
{
    gemm_job *j = (gemm_job *)arg;
    int64_t *cls = (int64_t *)malloc(sizeof(int64_t) * NSHIFT);
    unsigned char *used = (unsigned char *)malloc(NSHIFT);
    int *used_list = (int *)malloc(sizeof(int) * NSHIFT);
    for (int m = j->row0; m < j->row1; m++) {
        for (int n = 0; n < j->N; n++) {
            memset(used, 0, NSHIFT);
            int nused = 0;
            quire_t q; q_zero(&q);
            for (int k = 0; k < j->K; k++) {
                uint32_t ca, cb;
                if (j->fmt_bits == 8) {
                    ca = ((const uint8_t *)j->A)[(size_t)m * j->K + k];
                    cb = ((const uint8_t *)j->B)[(size_t)n * j->K + k];
                } else {
                    ca = ((const uint16_t *)j->A)[(size_t)m * j->K + k];
                    cb = ((const uint16_t *)j->B)[(size_t)n * j->K + k];
                }
                int64_t P = j->mA[ca] * j->mA[cb];
                if (P == 0) continue;
                int sh = j->eA[ca] + j->eA[cb] + QFRAC;
                if (j->sa) sh += j->sa[(size_t)m * j->G + k / j->group];
                if (j->sb) sh += j->sb[(size_t)n * j->G + k / j->group];
                if (sh >= 0) {
                    int idx = sh - SHIFT_MIN;
                    if (!used[idx]) { used[idx] = 1; cls[idx] = 0; used_list[nused++] = idx; }
                    cls[idx] += P;
                } else {
                    int r = -sh;
                    int64_t t;
                    if (r >= 63) t = 0;
                    else t = P < 0 ? -((-P) >> r) : (P >> r);   /* trunc toward zero */
                    q_add_shifted(&q, t, 0);
                }
            }
            for (int u = 0; u < nused; u++) {
                int idx = used_list[u];
                if (cls[idx]) q_add_shifted(&q, cls[idx], idx + SHIFT_MIN);
            }
            size_t o = (size_t)m * j->N + n;
            if (j->out_bp32) j->out_bp32[o] = q_to_bp32(&q);
            if (j->out_quire) memcpy(j->out_quire + o * (size_t)j->nlimbs, q.w, sizeof(uint32_t) * (size_t)j->nlimbs);
        }
    }
    free(cls); free(used); free(used_list);
    return NULL;
}

/* fmt_bits: 8 (bp8 codes, uint8) or 16 (bp16 codes, uint16).
 * sa / sb: per-(row, group) exponents [rows, ceil(K/group)] or NULL.
 * out_quire: optional [M, N, nlimbs] little-endian 32-bit limbs (truncated
 * two's complement).  Returns 0, or -1 on bad arguments. */
int orc_quire_gemm(int fmt_bits, const void *A, const void *B, int M, int N, int K,
                   const int32_t *sa, const int32_t *sb, int group,
                   uint32_t *out_bp32, uint32_t *out_quire, int nlimbs, int nthreads)
{
    if (fmt_bits != 8 && fmt_bits != 16) return -1;
    if (M < 0 || N < 0 || K < 0) return -1;
    if ((sa || sb) && group <= 0) return -1;
    if (out_quire && (nlimbs < 1 || nlimbs > QL)) return -1;
    int ncode = 1 << fmt_bits;
    int64_t *mt = (int64_t *)malloc(sizeof(int64_t) * ncode);
    int *et = (int *)malloc(sizeof(int) * ncode);
    for (int c = 0; c < ncode; c++) orc_decode_me(fmt_bits, (uint32_t)c, &mt[c], &et[c]);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > M && M > 0) nthreads = M;
    if (M == 0 || N == 0) { free(mt); free(et); return 0; }
    gemm_job *jobs = (gemm_job *)calloc((size_t)nthreads, sizeof(gemm_job));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    int G = group > 0 ? (K + group - 1) / group : 1;
    for (int t = 0; t < nthreads; t++) {
        gemm_job *j = &jobs[t];
        j->fmt_bits = fmt_bits; j->M = M; j->N = N; j->K = K; j->group = group > 0 ? group : 1; j->G = G;
        j->A = A; j->B = B; j->sa = sa; j->sb = sb;
        j->out_bp32 = out_bp32; j->out_quire = out_quire; j->nlimbs = nlimbs;
        j->row0 = (int)((int64_t)M * t / nthreads);
        j->row1 = (int)((int64_t)M * (t + 1) / nthreads);
        j->mA = mt; j->eA = et;
    }
    for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, gemm_worker, &jobs[t]);
    gemm_worker(&jobs[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(jobs); free(th); free(mt); free(et);
    return 0;
}

/* bp32 decode to double (reference/bposit_ref.py:43-94); NaR -> NaN. */
double orc_bp32_to_double(uint32_t code)
{
    return decode_double(32, code);
}

void orc_bp32_to_double_batch(const uint32_t *codes, size_t n, double *out)
{
    for (size_t i = 0; i < n; i++) out[i] = decode_double(32, codes[i]);
}

/* bp8 truncating encode of an exact value (reference/bposit_ref.py:216-270
 * on Fraction(x), i.e. without limit_denominator). */
static uint32_t encode_unsigned8(double value)
{
    if (value == 0) return 0;
    int total_e = 0;
    double v = value;
    if (v >= 1) { while (v >= 2) { v /= 2; total_e++; } }
    else { while (v < 1) { v *= 2; total_e--; } }
    if (total_e > 24) return 0x7F;
    if (total_e < -24) return 0x01;
    int k = total_e >> 2, e = total_e & 3;
    double f = v - 1;
    int bits[24]; int nb = 0;
    if (k >= 0) { for (int i = 0; i < k + 1; i++) bits[nb++] = 1; bits[nb++] = 0; }
    else { for (int i = 0; i < -k; i++) bits[nb++] = 0; bits[nb++] = 1; }
    if (nb >= 7) nb = 7;
    else {
        for (int i = 1; i >= 0; i--) { bits[nb++] = (e >> i) & 1; if (nb == 7) break; }
        while (nb < 8) { f *= 2; if (f >= 1) { bits[nb++] = 1; f -= 1; } else bits[nb++] = 0; }
        if (nb > 7) nb = 7;
    }
    uint32_t out = 0;
    for (int i = 0; i < nb; i++) out = (out << 1) | (uint32_t)bits[i];
    out <<= (7 - nb);
    return out & 0x7F;
}

uint8_t orc_encode_bp8_exact(double x)
{
    if (x == 0 || isnan(x)) return isnan(x) ? 0x80 : 0;
    int sign = x < 0;
    uint32_t f = isinf(x) ? 0x7F : encode_unsigned8(fabs(x));
    if (sign) f = ((~f) + 1u) & 0x7F;
    return (uint8_t)((sign << 7) | f);
}
