// bp_gemm_common.cuh -- device helpers shared by the quire GEMM paths and the
// standalone quire->bp32 kernel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_format.cuh"

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
// bit `base` (units of 2^-96): the bp32 code and, optionally, `nlimbs` limbs of
// the raw quire (two's complement, truncated to nlimbs*32 bits).
__device__ __forceinline__ void write_fast_output(unsigned __int128 acc, int base, uint32_t *ob,
                                                  uint32_t *oq, int nlimbs) {
  bool neg = (uint64_t)(acc >> 127) != 0u;
  unsigned __int128 mag = neg ? (unsigned __int128)0 - acc : acc;
  *ob = bp32_from_mag(neg, (uint64_t)(mag >> 64), (uint64_t)mag, base - 96);
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
}

}  // namespace bp
