// bp_gemm_common.cuh -- device helpers shared by the quire GEMM paths and the
// standalone quire->bp32 kernel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_format.cuh"
#include "bp_internal.cuh"

namespace bp {

// quire256_to_bposit32 on a little-endian two's complement quire of NL 32-bit
// limbs (96 fraction bits).  Only the 64 bits below the magnitude's msb can
// reach a bp32 field, so the magnitude is reduced to that window.
template <int NL>
__device__ __forceinline__ uint32_t bp32_from_limbs(const uint32_t *q) {
  bool neg = (q[NL - 1] >> 31) != 0u;
  uint32_t m[NL];
  uint64_t carry = neg ? 1u : 0u;
#pragma unroll
  for (int i = 0; i < NL; ++i) {
    uint64_t v = (uint64_t)(neg ? ~q[i] : q[i]) + carry;
    m[i] = (uint32_t)v;
    carry = v >> 32;
  }
  int top = -1;
#pragma unroll
  for (int i = 0; i < NL; ++i)
    if (m[i]) top = i;
  if (top < 0) return 0u;
  uint32_t mt = 0u;
#pragma unroll
  for (int i = 0; i < NL; ++i)
    if (i == top) mt = m[i];
  int msb = 32 * top + 31 - __clz((int)mt);
  uint64_t w = 0;
#pragma unroll
  for (int i = 0; i < NL; ++i) {
    int off = 32 * i - (msb - 63);   // position of limb i's bit 0 inside the window
    if (off >= 64 || off <= -32) continue;
    uint64_t v = m[i];
    w |= off >= 0 ? (v << off) : (v >> (-off));
  }
  return bp32_from_mag(neg, 0u, w, (msb - 63) - 96);
}

__device__ __forceinline__ uint32_t bp32_from_limbs16(const uint32_t *q) { return bp32_from_limbs<16>(q); }

__device__ __forceinline__ int ceil_log2_int(int K) {
  return K <= 1 ? 0 : 32 - __clz(K - 1);
}

// Bits (sign included) of the narrowest two's complement window that holds
// every partial sum of a dot product between rows with stats ra / rb:
// x = {min lsb exponent, max binade, nonzero, -}.
__device__ __forceinline__ int fast_width(int4 ra, int4 rb, int K, int) {
  return (ra.y + rb.y + 2) - (ra.x + rb.x) + ceil_log2_int(K) + 1;
}

// Writes one output from an exact 128-bit sum `acc` whose bit 0 sits at quire
// bit `base` (units of 2^-96): the bp32 code (returned, and stored at `ob`
// unless it is null) and, optionally, `nlimbs` limbs of the raw quire (two's
// complement, truncated to nlimbs*32 bits).
__device__ __forceinline__ uint32_t write_fast_output(unsigned __int128 acc, int base, uint32_t *ob,
                                                      uint32_t *oq, int nlimbs) {
  bool neg = (uint64_t)(acc >> 127) != 0u;
  unsigned __int128 mag = neg ? (unsigned __int128)0 - acc : acc;
  const uint32_t code = bp32_from_mag(neg, (uint64_t)(mag >> 64), (uint64_t)mag, base - 96);
  if (ob) *ob = code;
  if (oq) {
    for (int i = 0; i < nlimbs; ++i) {
      int o = 32 * i - base;
      uint32_t v;
      if (o <= -32) v = 0u;
      else if (o < 0) v = (uint32_t)(acc << (-o));
      else if (o < 128) v = (uint32_t)((unsigned __int128)((__int128)acc >> o));
      else v = neg ? 0xFFFFFFFFu : 0u;
      oq[i] = v;
    }
  }
  return code;
}

// 2^e as a double, for e in the normal range [-1022, 1023] (built from its bits).
__device__ __forceinline__ double pow2d(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

// Exact value of a bp32 code times 2^extra (NaR -> 0.0 like _bp32_to_float,
// reference/bposit_quantize.py:66-68): one multiply by an exact power of two
// while that is a normal double, scalbn (which rounds subnormals and
// overflows as IEEE does) beyond.
__device__ __forceinline__ double bp32_value_scaled(uint32_t code, int extra) {
  Dec d = decode_posit<32, 3>(code);
  if (d.kind != 0) return 0.0;
  const int e = d.scale - d.fw + extra;
  const double m = (double)((1u << d.fw) + d.fbits);
  const double v = (e >= -1022 && e <= 1023) ? m * pow2d(e) : scalbn(m, e);
  return d.sign ? -v : v;
}

// The fp32 hand-off of one output: value(code) * 2^extra (exact in float64)
// plus bias, added in float64 and rounded to the nearest-even fp32 -- the same
// two steps as the oracle's float64 rescale followed by astype(float32).
// NaR -> NaN.
__device__ __forceinline__ float bp32_f32_out(uint32_t code, int extra, float bias) {
  const double v = bp32_value_scaled(code, extra) + (double)bias;
  return code == 0x80000000u ? __uint_as_float(0x7FC00000u) : __double2float_rn(v);
}

// Stores output (i, j)'s bposit32 code and, when requested, its fp32 hand-off.
__device__ __forceinline__ void store_output(const GemmArgs &a, int i, int j, uint32_t code) {
  if (a.out) a.out[(size_t)i * a.ldo + j] = code;
  if (a.out_f32)
    a.out_f32[(size_t)i * a.ldf + j] =
        bp32_f32_out(code, (a.re ? a.re[i] : 0) + (a.ce ? a.ce[j] : 0), a.bias ? a.bias[j] : 0.0f);
}

// ---- exact per-element form and the slow (512-bit, per-term truncating) path ----
struct ElemME {
  int m;   // signed mantissa (0 for zero / NaR)
  int e;   // exponent of the mantissa's bit 0, group scale included
};

template <int FMT>
__device__ __forceinline__ ElemME load_elem(const void *base, int row, int K, int k,
                                            const int32_t *s, int G, int group) {
  uint32_t c = FMT == 8 ? ((const uint8_t *)base)[(size_t)row * K + k]
                        : ((const uint16_t *)base)[(size_t)row * K + k];
  ElemME r;
  if (FMT == 8) posit_to_me<8, 2>(c, r.m, r.e);
  else posit_to_me<16, 3>(c, r.m, r.e);
  if (s && r.m) r.e += s[(size_t)row * G + k / group];
  return r;
}

// 512-bit two's complement quire in 16 limbs: q += v * 2^sh (sh >= 0).
__device__ inline void q512_add(uint32_t *q, int64_t v, int sh) {
  if (v == 0 || sh >= 512) return;
  int limb = sh >> 5, bit = sh & 31;
  uint64_t uv = (uint64_t)v;
  uint32_t fill = v < 0 ? 0xFFFFFFFFu : 0u;
  uint32_t lo = (uint32_t)uv, hi = (uint32_t)(uv >> 32);
  uint32_t x0 = bit ? lo << bit : lo;
  uint32_t x1 = bit ? (hi << bit) | (lo >> (32 - bit)) : hi;
  uint32_t x2 = bit ? (fill << bit) | (hi >> (32 - bit)) : fill;
  uint64_t carry = 0;
  for (int i = limb; i < 16; ++i) {
    uint32_t t = i == limb ? x0 : (i == limb + 1 ? x1 : (i == limb + 2 ? x2 : fill));
    uint64_t sum = (uint64_t)q[i] + t + carry;
    q[i] = (uint32_t)sum;
    carry = sum >> 32;
  }
}

template <int FMT>
__device__ inline void slow_output(const GemmArgs &a, int m, int n, uint32_t *out_bp32, uint32_t *out_q) {
  uint32_t q[16];
  for (int i = 0; i < 16; ++i) q[i] = 0u;
  for (int k = 0; k < a.K; ++k) {
    ElemME x = load_elem<FMT>(a.A, m, a.K, k, a.sa, a.G, a.group);
    ElemME y = load_elem<FMT>(a.B, n, a.K, k, a.sb, a.G, a.group);
    int64_t P = (int64_t)x.m * y.m;
    if (!P) continue;
    int sh = x.e + y.e + 96;
    if (sh >= 0) {
      q512_add(q, P, sh);
    } else {
      int r = -sh;
      int64_t t = r >= 63 ? 0 : (P < 0 ? -((-P) >> r) : (P >> r));   // trunc toward zero
      q512_add(q, t, 0);
    }
  }
  *out_bp32 = bp32_from_limbs16(q);
  if (out_q)
    for (int i = 0; i < a.nlimbs; ++i) out_q[i] = q[i];
}

}  // namespace bp
