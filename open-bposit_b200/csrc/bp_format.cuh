// bp_format.cuh -- b-posit bit-level format helpers shared by host and device.
//
// Formats (reference/bposit_ref.py): bp8 = 8-bit posit, eS=2 (useed 16, values
// 2^-24..2^24); bp16 = 16-bit, eS=3 (useed 256, 2^-112..2^112); bp32 = 32-bit,
// eS=3.  Decoding follows the regime run-length rule of decode_bposit8/16/32
// (reference/bposit_ref.py:162-193, 306-355, 43-74): two's complement of the
// trailing bits for negatives, exponent left-padded when the regime leaves
// fewer than eS bits.  Every helper here is integer-only.
#pragma once
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define BP_HD __host__ __device__ __forceinline__
#else
#define BP_HD inline
#endif

namespace bp {

BP_HD int clz32(uint32_t x) {
#ifdef __CUDA_ARCH__
  return __clz((int)x);
#else
  return x ? __builtin_clz(x) : 32;
#endif
}
BP_HD int clz64(uint64_t x) {
#ifdef __CUDA_ARCH__
  return __clzll((long long)x);
#else
  return x ? __builtin_clzll(x) : 64;
#endif
}

// Decoded posit: kind 0 = finite nonzero, 1 = zero, 2 = NaR.  For finite values
// |value| = (2^fw + fbits) * 2^(scale - fw), scale = k*2^eS + e is the binade.
struct Dec {
  int kind;
  int sign;
  int scale;
  int fw;
  uint32_t fbits;
};

template <int NB, int ES>
BP_HD Dec decode_posit(uint32_t p) {
  const uint32_t sbit = 1u << (NB - 1);
  const uint32_t fmask = sbit - 1u;
  const uint32_t mask = (NB == 32) ? 0xFFFFFFFFu : ((sbit << 1) - 1u);
  p &= mask;
  Dec d{0, 0, 0, 0, 0u};
  if (p == 0u) { d.kind = 1; return d; }
  if (p == sbit) { d.kind = 2; return d; }
  d.sign = (int)(p >> (NB - 1));
  uint32_t rest = p & fmask;
  if (d.sign) rest = (0u - rest) & fmask;
  uint32_t al = rest << (33 - NB);          // field MSB at bit 31, zero padding below
  int lead = (int)(al >> 31);
  uint32_t inv = lead ? ~al : al;           // count the run of `lead` bits
  int rs = clz32(inv);
  if (rs > NB - 1) rs = NB - 1;
  int k = lead ? rs - 1 : -rs;
  int rem = NB - 2 - rs;                    // bits after regime + terminator
  int e = 0, fw = 0;
  uint32_t fb = 0;
  if (rem > 0) {
    uint32_t rest2 = rest & ((1u << rem) - 1u);
    int ew = rem < ES ? rem : ES;
    e = (int)((rest2 >> (rem - ew)) << (ES - ew));
    fw = rem - ew;
    fb = rest2 & ((1u << fw) - 1u);
  }
  d.scale = k * (1 << ES) + e;
  d.fw = fw;
  d.fbits = fb;
  return d;
}

// fp32 bit pattern of a bp8 / bp16 code (exact: |scale| <= 112 keeps it a
// normal float).  Zero and NaR give +0.0 (code_value semantics,
// reference/bposit_ref.py:1022-1025).
template <int NB, int ES>
BP_HD uint32_t posit_to_f32_bits(uint32_t code) {
  Dec d = decode_posit<NB, ES>(code);
  if (d.kind != 0) return 0u;
  return ((uint32_t)d.sign << 31) | ((uint32_t)(d.scale + 127) << 23) | (d.fbits << (23 - d.fw));
}

// Exact integer form: value = mant * 2^exp, |mant| = 2^fw + fbits (unreduced,
// the form of the bp8 decode ROM in reference/gen_rtl_vectors.py:289-298).
template <int NB, int ES>
BP_HD void posit_to_me(uint32_t code, int &mant, int &exp) {
  Dec d = decode_posit<NB, ES>(code);
  if (d.kind != 0) { mant = 0; exp = 0; return; }
  int m = (1 << d.fw) + (int)d.fbits;
  mant = d.sign ? -m : m;
  exp = d.scale - d.fw;
}

// ---------------------------------------------------------------------------
// bp8 code of the largest grid value <= 2^E, for E in [-24, 24] (the
// truncating encode of reference/bposit_ref.py:216-255 applied to 2^E).
// ---------------------------------------------------------------------------
BP_HD uint32_t bp8_trunc_pow2(int E) {
  int k = E >> 2;                 // arithmetic shift = floor division
  int e = E & 3;
  int rl = k >= 0 ? k + 2 : 1 - k;
  if (rl >= 7) {
    if (k >= 0) return k >= 5 ? (k >= 6 ? 0x7Fu : 0x7Eu) : 0u;
    return 0x01u;
  }
  int avail = 7 - rl;
  int eb = avail < 2 ? avail : 2;
  int fw = avail - eb;
  uint32_t R = k >= 0 ? (((1u << (k + 1)) - 1u) << 1) : 1u;
  return (R << avail) | ((uint32_t)(e >> (2 - eb)) << fw);
}

// Quantize table for fp32 -> bp8, indexed by the biased fp32 exponent b of |x|:
//   mag = c_lo + (M >> sh) + ((M & ((1 << sh) - 1)) > thr)
// with M the 23-bit fp32 mantissa.  This reproduces bposit_fast.quantize_bp8
// (reference/bposit_fast.py:69-99): nearest=True counts the midpoints
// (g[i] + g[i+1]) / 2 strictly below |x| (so ties go to the lower magnitude),
// nearest=False takes the largest grid value <= |x|, and both send any nonzero
// |x| below minpos to minpos.  `never` = 0x7FFFFF (M never exceeds it).
struct QEntry {
  uint32_t lo_sh;   // c_lo | sh << 8
  uint32_t thr;
};

BP_HD double bp8_value_f64(uint32_t code) {
  Dec d = decode_posit<8, 2>(code);
  if (d.kind != 0) return 0.0;
  double v = (double)((1u << d.fw) + d.fbits);
  int s = d.scale - d.fw;
  // exact power-of-two scaling without libm
  while (s > 0) { v *= 2.0; --s; }
  while (s < 0) { v *= 0.5; ++s; }
  return d.sign ? -v : v;
}

BP_HD QEntry bp8_qentry(int b, bool nearest) {
  const uint32_t never = 0x7FFFFFu;
  QEntry q;
  if (b == 0) { q.lo_sh = 0u | (23u << 8); q.thr = 0u; return q; }     // zero / subnormal
  int E = b - 127;
  if (b == 255 || E >= 24) { q.lo_sh = 127u | (23u << 8); q.thr = never; return q; }
  if (E < -24) { q.lo_sh = 1u | (23u << 8); q.thr = never; return q; }
  uint32_t clo = bp8_trunc_pow2(E);
  double P = 1.0;
  for (int i = 0; i < (E > 0 ? E : -E); ++i) P = E > 0 ? P * 2.0 : P * 0.5;
  double glo = bp8_value_f64(clo);
  double ghi = bp8_value_f64(clo + 1u);
  if (glo == P && ghi < 2.0 * P) {
    // regular binade: grid points P * (1 + j / 2^fw), j < 2^fw
    double sp = ghi - glo;
    int fw = 0;
    while (sp * (double)(1 << fw) < P) ++fw;
    uint32_t sh = 23u - (uint32_t)fw;
    q.lo_sh = clo | (sh << 8);
    q.thr = nearest ? (1u << (sh - 1)) : never;
    return q;
  }
  // at most one grid point in the binade: compare with the midpoint directly
  q.lo_sh = clo | (23u << 8);
  if (!nearest) { q.thr = never; return q; }
  double mid = (glo + ghi) * 0.5;
  if (mid >= 2.0 * P) { q.thr = never; return q; }
  double t = (mid / P - 1.0) * 8388608.0;   // exact: mid is dyadic with few bits
  q.thr = (uint32_t)t;
  return q;
}

// Apply a quantize entry to |x| given as (M, table entry); returns the 7-bit
// magnitude code (0 only for x == 0).
BP_HD uint32_t bp8_apply(QEntry q, uint32_t M) {
  uint32_t sh = q.lo_sh >> 8;
  uint32_t mask = (1u << sh) - 1u;
  return (q.lo_sh & 0xFFu) + (M >> sh) + ((M & mask) > q.thr ? 1u : 0u);
}

// ---------------------------------------------------------------------------
// fp32 -> bp16, the bit-string encoder _encode_unsigned(value, mode) of
// reference/bposit_ref.py:382-486 on the exact value of x: regime, up to three
// exponent bits, fraction bits, then (rtne) round up when the first dropped
// fraction bit is set and (any later bit is set or the kept LSB is odd),
// saturating at maxpos.  When the regime leaves no room for all exponent bits
// the first dropped bit is still the first FRACTION bit, as in the reference.
// NaN -> NaR (0x8000) and +-inf -> +-maxpos are extensions for inputs the
// reference rejects.
// ---------------------------------------------------------------------------
BP_HD uint32_t bp16_encode_bits(uint32_t u, bool rtne) {
  uint32_t sign = u >> 31;
  uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x8000u;
  if (a == 0u) return 0u;
  uint32_t field;
  int b = (int)(a >> 23);
  uint32_t M = a & 0x7FFFFFu;
  int E = b - 127;
  if (b == 0 || E < -112) field = 0x0001u;
  else if (b == 255 || E > 112) field = 0x7FFFu;
  else {
    int k = E >> 3, e = E & 7;
    int rl = k >= 0 ? k + 2 : 1 - k;
    if (rl >= 15) {
      field = k >= 0 ? (k >= 14 ? 0x7FFFu : 0x7FFEu) : 0x0001u;
    } else {
      int avail = 15 - rl;
      int eb = avail < 3 ? avail : 3;
      int fb = avail - eb;
      uint32_t R = k >= 0 ? (((1u << (k + 1)) - 1u) << 1) : 1u;
      field = (R << avail) | ((uint32_t)(e >> (3 - eb)) << fb) | (M >> (23 - fb));
      if (rtne) {
        uint32_t rbit = (M >> (22 - fb)) & 1u;
        uint32_t sticky = M & ((1u << (22 - fb)) - 1u);
        bool up = rbit && (sticky != 0u || (field & 1u));
        if (up && field < 0x7FFFu) field += 1u;
      }
    }
  }
  if (sign) field = (0u - field) & 0x7FFFu;
  return (sign << 15) | field;
}

// The same encoder as a per-binade table, for the streaming kernels.  Inside
// one fp32 binade b (biased exponent) the regime and exponent bits are fixed,
// so the 15-bit field is base(b) + (M >> sh(b)) with M the 23-bit mantissa,
// sh = 23 - (fraction bits kept); binades whose field is a constant (zero and
// subnormal inputs -> minpos, beyond +-2^112 or a regime of 15 bits -> the
// saturated field) use sh = 24, which keeps no mantissa bit and never rounds.
// Round to nearest even on the field: with half = 2^(sh-1) the rounded field
// is base + ((M + half - 1 + lsb) >> sh), lsb = the truncated field's lowest
// bit -- the rbit && (sticky || odd) rule of bp16_encode_bits, including its
// quirk that with fewer than three exponent bits kept (sh = 23) the round bit
// is the first fraction bit.  In the normal binades the field stays below
// 0x7FFE before rounding, so the reference's saturation check never fires.
// Entry: lo = base | sh << 16, hm1 = half - 1 (0 for truncation).
BP_HD void bp16_qentry(int b, bool rtne, uint32_t &lo, uint32_t &hm1) {
  uint32_t base, sh = 24u;
  const int E = b - 127;
  if (b == 0 || E < -112) base = 0x0001u;
  else if (b == 255 || E > 112) base = 0x7FFFu;
  else {
    const int k = E >> 3, e = E & 7;
    const int rl = k >= 0 ? k + 2 : 1 - k;
    if (rl >= 15) {
      base = k >= 0 ? (k >= 14 ? 0x7FFFu : 0x7FFEu) : 0x0001u;
    } else {
      const int avail = 15 - rl;
      const int eb = avail < 3 ? avail : 3;
      const int fb = avail - eb;
      const uint32_t R = k >= 0 ? (((1u << (k + 1)) - 1u) << 1) : 1u;
      base = (R << avail) | ((uint32_t)(e >> (3 - eb)) << fb);
      sh = 23u - (uint32_t)fb;
    }
  }
  lo = base | (sh << 16);
  hm1 = rtne ? (1u << (sh - 1u)) - 1u : 0u;
}

// Code of fp32 bits u from its binade's entry (bp16_qentry of (u >> 23) & 0xFF):
// identical to bp16_encode_bits(u, rtne).
BP_HD uint32_t bp16_encode_tbl(uint32_t u, uint32_t lo, uint32_t hm1, bool rtne) {
  const uint32_t a = u & 0x7FFFFFFFu;
  const uint32_t M = a & 0x7FFFFFu;
  const uint32_t base = lo & 0xFFFFu, sh = lo >> 16;
  uint32_t field = base + (M >> sh);
  if (rtne) field = base + ((M + hm1 + (field & 1u)) >> sh);
  uint32_t code = (u >> 31) ? (0x8000u | ((0u - field) & 0x7FFFu)) : field;
  code = a == 0u ? 0u : code;
  return a > 0x7F800000u ? 0x8000u : code;
}

// fp32 bit pattern of a bp16 code (posit_to_f32_bits<16, 3> in closed form):
// the 15-bit field is left-aligned at bit 31, the regime run r is counted with
// one clz, and shifting the field past the regime and its terminator leaves
// the three exponent bits and then the fraction at the top of the word (the
// bits the regime leaves no room for shift in as zeros).  Zero and NaR -> +0.0.
BP_HD uint32_t bp16_to_f32_bits(uint32_t c) {
  const uint32_t neg = (c >> 15) & 1u;
  const uint32_t f = (neg ? (0u - c) : c) & 0x7FFFu;
  const uint32_t al = f << 17;
  const uint32_t inv = al ^ (uint32_t)((int32_t)al >> 31);
  int r = clz32(inv);
  r = r > 15 ? 15 : r;
  const int k = (al >> 31) ? r - 1 : -r;
  const uint32_t x = al << (r + 1);                  // r <= 15
  const int scale = 8 * k + (int)(x >> 29);
  const uint32_t bits = (neg << 31) | ((uint32_t)(scale + 127) << 23) | ((x << 3) >> 9);
  return f ? bits : 0u;
}

// ---------------------------------------------------------------------------
// Signed streaming tables.  Indexed by u >> 23 (the sign and the biased
// exponent of the fp32 bits u), each entry gives a signed base code bs and a
// shift sh so that, with M the 23-bit mantissa, c the entry's rounding addend
// and q = (M + c) >> sh, the code is bs + q for positive x and bs - q for
// negative x (low 8 / 16 bits).  Negative entries hold 2^NB - base, so bs - q
// is the two's complement of the magnitude code base + q.  Zero, subnormal,
// inf and NaN inputs need no special case: their entries use sh = 23 and
// c = 2^23 - 1 (minus the RTNE parity bit for bp16), which makes q = 1 exactly
// when M != 0 -- zero -> code 0 (the -0 entry's 2^NB wraps to 0), subnormal ->
// +-minpos, inf -> +-maxpos and NaN -> maxpos + 1 = NaR.
// ---------------------------------------------------------------------------

// bp8 (bp8_qentry semantics).  x = bs | sh << 16; c = 2^sh - 1 - thr, the
// addend that carries into the code exactly when M's dropped bits exceed thr
// (0 for the truncating mode's "never").
BP_HD void bp8_qentry_signed(int idx, bool nearest, uint32_t &x, uint32_t &c) {
  const int b = idx & 0xFF;
  const bool neg = (idx >> 8) & 1;
  const QEntry q = bp8_qentry(b, nearest);
  const uint32_t base = q.lo_sh & 0xFFu, sh = q.lo_sh >> 8;
  c = q.thr >= 0x7FFFFFu ? 0u : (1u << sh) - 1u - q.thr;
  if (b == 255) c = 0x7FFFFFu;   // sh = 23: inf -> maxpos (127), NaN -> 128 = NaR
  x = (neg ? 0x100u - base : base) | (sh << 16);
}

BP_HD uint32_t bp8_encode_signed(uint32_t u, uint32_t x, uint32_t c) {
  const uint32_t q = ((u & 0x7FFFFFu) + c) >> (x >> 16);
  const uint32_t m = (uint32_t)((int32_t)u >> 31);
  return ((x & 0xFFFFu) + ((q ^ m) - m)) & 0xFFu;
}

// bp16 (bp16_qentry semantics, RTNE or truncating).  x = bs | sh << 17 (the
// -0 entry's bs is 0x10000, 17 bits); c = half - 1 for RTNE, 0 for
// truncation; with RTNE the parity of the truncated field, (bs ^ (M >> sh)) & 1,
// is added as well.
BP_HD void bp16_qentry_signed(int idx, bool rtne, uint32_t &x, uint32_t &c) {
  const int b = idx & 0xFF;
  const bool neg = (idx >> 8) & 1;
  uint32_t lo, hm1;
  bp16_qentry(b, rtne, lo, hm1);
  uint32_t base = lo & 0xFFFFu, sh = lo >> 16;
  c = hm1;
  if (b == 0) { base = 0u; sh = 23u; c = 0x7FFFFFu; }                          // 0 -> 0, subnormal -> minpos
  if (b == 255) { base = 0x7FFFu; sh = 23u; c = rtne ? 0x7FFFFEu : 0x7FFFFFu; }  // odd base: parity adds 1
  x = (neg ? 0x10000u - base : base) | (sh << 17);
}

template <bool RTNE>
BP_HD uint32_t bp16_encode_signed(uint32_t u, uint32_t x, uint32_t c) {
  const uint32_t M = u & 0x7FFFFFu, sh = x >> 17, bs = x & 0x1FFFFu;
  const uint32_t lsb = RTNE ? ((bs ^ (M >> sh)) & 1u) : 0u;
  const uint32_t q = (M + c + lsb) >> sh;
  const uint32_t m = (uint32_t)((int32_t)u >> 31);
  return (bs + ((q ^ m) - m)) & 0xFFFFu;
}

// The positive 15-bit field of a bp16 code (two's complement for negatives).
BP_HD uint32_t bp16_field(uint32_t c) { return (((c >> 15) & 1u) ? 0u - c : c) & 0x7FFFu; }

// ---------------------------------------------------------------------------
// bp32 from an exact magnitude: value = mag * 2^lsb_exp, mag = (hi:lo) 128-bit.
// The truncating bit-string encoder of reference/bposit_ref.py:97-150 as used
// by quire256_to_bposit32 (:703-722): total_e = floor(log2 value), regime,
// up to three exponent bits, then fraction bits, all cut at 31 bits; clamp at
// total_e beyond +-240; negatives take the two's complement of the field.
// ---------------------------------------------------------------------------
BP_HD uint32_t bp32_from_mag(bool neg, uint64_t hi, uint64_t lo, int lsb_exp) {
  if (hi == 0u && lo == 0u) return 0u;
  int msb = hi ? 127 - clz64(hi) : 63 - clz64(lo);
  int te = msb + lsb_exp;
  uint32_t field;
  if (te > 240) field = 0x7FFFFFFFu;
  else if (te < -240) field = 0x00000001u;
  else {
    int k = te >> 3, e = te & 7;
    int rl = k >= 0 ? k + 2 : 1 - k;
    if (rl >= 31) {
      field = k >= 0 ? (k >= 30 ? 0x7FFFFFFFu : 0x7FFFFFFEu) : 0x00000001u;
    } else {
      int avail = 31 - rl;
      int eb = avail < 3 ? avail : 3;
      int fb = avail - eb;
      uint32_t R = k >= 0 ? (((1u << (k + 1)) - 1u) << 1) : 1u;
      uint32_t f = 0u;
      if (fb > 0) {
        // 64-bit window whose bit 63 is the msb of mag
        uint64_t top;
        int s = 127 - msb;                       // left shift that puts msb at bit 127
        if (s >= 64) top = lo << (s - 64);
        else if (s == 0) top = hi;
        else top = (hi << s) | (lo >> (64 - s));
        f = (uint32_t)((top << 1) >> (64 - fb));
      }
      field = (R << avail) | ((uint32_t)(e >> (3 - eb)) << fb) | f;
    }
  }
  if (neg) field = (0u - field) & 0x7FFFFFFFu;
  return (neg ? 0x80000000u : 0u) | field;
}

// x >> s for any s >= 0 (0 once s >= 32), one funnel shift on the device.
BP_HD uint32_t shr_clamp(uint32_t x, int s) {
#ifdef __CUDA_ARCH__
  return __funnelshift_rc(x, 0u, (uint32_t)s);
#else
  return s >= 32 ? 0u : x >> s;
#endif
}

// Q as a double rounded toward zero (|Q| cut to 53 significant bits; exact
// below 2^53): the device's conversion instruction, emulated on the host.
BP_HD uint64_t i64_to_f64_rz_bits(long long Q) {
#ifdef __CUDA_ARCH__
  return (uint64_t)__double_as_longlong(__ll2double_rz(Q));
#else
  const bool neg = Q < 0;
  uint64_t m = neg ? 0ull - (uint64_t)Q : (uint64_t)Q;
  const int lz = clz64(m);
  if (lz < 11) m &= ~((1ull << (11 - lz)) - 1ull);   // keep 53 significant bits
  double d = (double)m;                              // now exact
  if (neg) d = -d;
  uint64_t b;
  memcpy(&b, &d, 8);
  return b;
#endif
}

// bp32_from_mag for a sum that fits a signed 64-bit integer: value Q * 2^lsb_exp,
// cut to the bposit32 bit string.  Q goes through one round-toward-zero
// conversion to double (a cut of |Q| to 53 bits, then the cut below to at most
// 27 bits: the same as one cut), which hands over the binade and the top
// fraction bits.  The regime, the three exponent bits and those fraction bits
// are laid out left-aligned in one 32-bit word W whose top 31 bits are the
// truncated field; te is clamped to regimes -30 .. 30, where W already reads
// maxpos (31 ones) or minpos (a single one in bit 1).  Selects only.
BP_HD uint32_t bp32_from_i64(long long Q, int lsb_exp) {
  const uint64_t bits = i64_to_f64_rz_bits(Q);
  const uint32_t hi = (uint32_t)(bits >> 32);
  const uint32_t f = (uint32_t)(bits >> 20);   // top 32 bits of the 52-bit fraction field
  int te = (int)((hi >> 20) & 0x7FFu) - 1023 + lsb_exp;
  te = te < -240 ? -240 : (te > 247 ? 247 : te);
  const int k = te >> 3, e = te & 7;
  const int rl = k >= 0 ? k + 2 : 1 - k;   // 2 .. 31
  const uint32_t R = k >= 0 ? (~0u << (31 - k)) : (1u << (31 + k));
  const uint32_t W = R | (((uint32_t)e << 29) >> rl) | shr_clamp(f, rl + 3);
  const uint32_t field = W >> 1;
  const uint32_t code = (hi >> 31) ? 0u - field : field;
  return Q ? code : 0u;
}

// The exact value of bp32_from_i64(Q, lsb_exp) as a double times 2^extra, for
// the sums whose bposit32 keeps all three exponent bits (regime of at most 28
// bits: total exponent in [-216, 215]), where that value is |Q| cut to its top
// 29 - rl bits: returns false for the others (and for Q = 0) so the caller can
// take the field route.  The double is exact (at most 27 significant bits);
// the scaling is an exponent add while the result stays a normal double.
BP_HD bool bp32_value_i64(long long Q, int lsb_exp, int extra, double &v) {
  if (Q == 0) return false;
  const bool neg = Q < 0;
  uint64_t m = neg ? 0ull - (uint64_t)Q : (uint64_t)Q;
  const int msb = 63 - clz64(m);
  const int te = msb + lsb_exp;
  const int k = te >> 3;
  const int rl = k >= 0 ? k + 2 : 1 - k;
  if (rl > 28) return false;
  const int drop = msb + 1 - (29 - rl);
  if (drop > 0) m &= ~((1ull << drop) - 1ull);
  const int e = lsb_exp + extra;
  // double(m) has exponent msb; the product stays normal for msb + e in [-1022, 1023]
  if (msb + e < -1022 || msb + e > 1023) return false;
  double d = (double)m;   // exact: at most 27 significant bits
  uint64_t b;
  memcpy(&b, &d, 8);
  b += (uint64_t)(int64_t)e << 52;
  memcpy(&d, &b, 8);
  v = neg ? -d : d;
  return true;
}

// ---- the small rungs: bposit4 (es 1, encode range 2^+-2) and AI-posit5
// (es 1, 2^+-4) (reference/bposit_ref.py:879-940) --------------------------
// Fraction(x).limit_denominator(10**8) is 0 exactly when |x| < 1/(2*10**8);
// this is the largest double below that bound (the float entry of the
// truncating encoders, reference/bposit_ref.py:258-270, 852-856).
#define BP_LIMIT_ZERO 0x1.5798ee2308c39p-28

// Truncating encode of a double with the reference's generic
// _encode_unsigned_gen + _encode_gen (reference/bposit_ref.py:806-866):
// floor(log2|x|) above MAXE -> maxpos, below -MAXE -> minpos, else regime,
// ES exponent bits (MSB first) and fraction bits cut to the NB-1 bit field;
// negative values take the field's two's complement.  NaN -> NaR.
template <int NB, int ES, int MAXE>
BP_HD uint32_t small_encode(double x) {
  constexpr int F = NB - 1;
  constexpr uint32_t fmask = (1u << F) - 1u;
  if (x != x) return 1u << F;
  const bool neg = x < 0.0;
  const double a = neg ? -x : x;
  if (a <= BP_LIMIT_ZERO) return 0u;
  uint32_t field;
  uint64_t u;
  memcpy(&u, &a, 8);
  const int be = (int)((u >> 52) & 0x7FF);
  if (be == 0x7FF) {
    field = fmask;                      // +-inf
  } else {
    const int te = be - 1023;           // a >= 2^-28: normal, floor(log2 a) exact
    if (te > MAXE) field = fmask;
    else if (te < -MAXE) field = 1u;
    else {
      const int k = te >> ES, e = te & ((1 << ES) - 1);
      uint32_t bits = 0;
      int nb = 0;
      auto push = [&](uint32_t b) {
        if (nb < F) bits = (bits << 1) | b;
        ++nb;
      };
      if (k >= 0) {
        for (int i = 0; i <= k; ++i) push(1u);
        push(0u);
      } else {
        for (int i = 0; i < -k; ++i) push(0u);
        push(1u);
      }
      if (nb < F) {
        for (int i = ES - 1; i >= 0 && nb < F; --i) push((uint32_t)(e >> i) & 1u);
        for (int i = 51; i >= 0 && nb < F; --i) push((uint32_t)(u >> i) & 1u);   // fraction, truncated
      }
      const int kept = nb < F ? nb : F;
      field = (bits << (F - kept)) & fmask;
    }
  }
  if (neg) field = (0u - field) & fmask;
  return (neg ? 1u << F : 0u) | field;
}

// quire256_to_bposit16 from the bposit32 of the same quire.  Both rounds
// truncate (reference/bposit_ref.py:97-135 for bp32; 382-486, mode
// "truncate", for bp16) the same bit string -- regime, three exponent bits
// (es = 3 in both formats), fraction -- so the 15-bit bp16 field is the top 15
// bits of the 31-bit bp32 field.  The formats differ only where bp16
// saturates: total exponent above 112 already gives 15 leading ones; below
// -112 the top 15 bits are zero and bp16 returns minpos (never zero).
BP_HD uint16_t bp16_from_bp32(uint32_t c) {
  if (c == 0u) return 0;
  const bool neg = (c >> 31) != 0u;
  const uint32_t f32 = neg ? (0u - c) & 0x7FFFFFFFu : c & 0x7FFFFFFFu;
  uint32_t f16 = f32 >> 16;
  if (f16 == 0u) f16 = 1u;
  return (uint16_t)(neg ? 0x8000u | ((0u - f16) & 0x7FFFu) : f16);
}

}  // namespace bp
