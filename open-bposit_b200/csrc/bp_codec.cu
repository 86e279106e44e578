// bp_codec.cu -- elementwise b-posit codec kernels (HBM-bound).
//
//  * decode: code -> exact fp32 value (bp8 via a 256-entry shared-memory LUT,
//    bp16 arithmetically), replacing code_value / bposit_fast._lut
//    (reference/bposit_ref.py:1022-1025, reference/bposit_fast.py:27-43).
//  * quantize_bp8: fp32 -> bp8 code (+ optional exact fp32 value),
//    bposit_fast.quantize_bp8(x, nearest=True|False) (reference/bposit_fast.py:69-99)
//    through the per-binade table of bp_format.cuh.
//  * encode_bp16: fp32 -> bp16, encode_bposit16(Fraction(x), "rtne"|"truncate")
//    (reference/bposit_ref.py:382-507).
//  * group_quantize_bp8: per-(row, group) power-of-two scale
//    2^ceil(log2(absmax / 2^24)) folded into the exponent, then quantize_bp8.
//  * quire_to_bp32: quire256_to_bposit32 (reference/bposit_ref.py:703-722).
//
// Layout: flat arrays.  The streaming kernels move units of four elements (a
// float4 of fp32 on one side, 4 or 8 bytes of codes on the other) in tiles
// whose every warp instruction touches one contiguous span, several loads in
// flight per thread; misaligned pointers and the last few elements take a
// scalar loop.  Grids are one block per tile (decode) or a multiple of the SM
// count (the encoders, grid-stride).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "bp_gemm_common.cuh"
#include "bp_internal.cuh"

namespace bp {
namespace {

constexpr int kThreads = 256;

inline int grid_for(size_t work_items, int per_sm = 8) {
  size_t want = (work_items + kThreads - 1) / kThreads;
  size_t cap = (size_t)sm_count() * per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

// ---------------------------------------------------------------- decode ---
// Tiles of kThreads * U vector units per block step: unit t + j * kThreads of
// a tile goes to thread t, so every load and every store instruction of a warp
// covers one contiguous span (a word of 4 bp8 codes or 4 bp16 codes in, a
// float4 out).  The U loads of a step are issued before any store.  The grid
// is one block per tile (no grid-stride for the vector part); elements past
// the last whole unit, and every element of a misaligned call, take the
// scalar loop.
template <int U>
__global__ void __launch_bounds__(kThreads) k_decode_bp8(const uint8_t *__restrict__ codes, size_t n,
                                                         float *__restrict__ out, bool vec) {
  __shared__ uint32_t lut[256];
  lut[threadIdx.x] = posit_to_f32_bits<8, 2>(threadIdx.x);
  __syncthreads();
  const size_t nw = vec ? n / 4 : 0;
  const uint32_t *w = reinterpret_cast<const uint32_t *>(codes);
  uint4 *o4 = reinterpret_cast<uint4 *>(out);
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = blockIdx.x * tile; base < nw; base += (size_t)gridDim.x * tile) {
    uint32_t v[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      v[j] = i < nw ? __ldcs(w + i) : 0u;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      if (i < nw)
        __stcs(o4 + i, make_uint4(lut[v[j] & 0xFFu], lut[(v[j] >> 8) & 0xFFu], lut[(v[j] >> 16) & 0xFFu],
                                  lut[v[j] >> 24]));
    }
  }
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = nw * 4 + tid; i < n; i += stride) out[i] = __uint_as_float(lut[codes[i]]);
}

// bp16: the fp32 pattern of every positive 15-bit field in a 32,768-entry
// table (128 KB of shared memory, built once per block from the closed form);
// a code costs one table load and a sign fix-up, whatever its regime length.
// One 1024-thread block per SM, grid-stride over tiles; four codes (8 bytes)
// per unit.
constexpr int kDec16Threads = 1024;
constexpr size_t kDec16Smem = (size_t)32768 * sizeof(uint32_t);

template <int U>
__global__ void __launch_bounds__(kDec16Threads, 1) k_decode_bp16(const uint16_t *__restrict__ codes, size_t n,
                                                                  float *__restrict__ out, bool vec) {
  extern __shared__ uint32_t lut16[];
  for (int f = threadIdx.x; f < 32768; f += kDec16Threads) lut16[f] = bp16_to_f32_bits((uint32_t)f);
  __syncthreads();
  auto dec = [&](uint32_t c) {
    const uint32_t f = bp16_field(c);
    return f ? (lut16[f] | ((c & 0x8000u) << 16)) : 0u;
  };
  const size_t nq = vec ? n / 4 : 0;
  const uint2 *c2 = reinterpret_cast<const uint2 *>(codes);
  uint4 *o4 = reinterpret_cast<uint4 *>(out);
  const size_t tile = (size_t)kDec16Threads * U;
  for (size_t base = blockIdx.x * tile; base < nq; base += (size_t)gridDim.x * tile) {
    uint2 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kDec16Threads;
      v[j] = i < nq ? __ldcs(c2 + i) : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kDec16Threads;
      if (i < nq)
        __stcs(o4 + i, make_uint4(dec(v[j].x & 0xFFFFu), dec(v[j].x >> 16), dec(v[j].y & 0xFFFFu), dec(v[j].y >> 16)));
    }
  }
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = nq * 4 + tid; i < n; i += stride) out[i] = __uint_as_float(dec(codes[i]));
}

// ------------------------------------------------------------ quantize bp8 ---
// Signed per-binade table (bp8_qentry_signed, 512 entries indexed by the sign
// and biased exponent): a code is one table load, a shift-add and a
// conditional negate (bp8_encode_signed), with zero, subnormals, inf and NaN
// folded into their entries.  Units of four elements (a float4 in, a word of
// codes out, and with `vals` a float4 of exact values) in the decode kernels'
// tile order; grid-stride over tiles, 8 blocks per SM.
template <bool NEAREST, bool VALUES, int U>
__global__ void __launch_bounds__(kThreads) k_quantize_bp8(const float *__restrict__ x, size_t n,
                                                           uint8_t *__restrict__ codes,
                                                           float *__restrict__ vals, bool vec) {
  __shared__ uint2 tbl[512];
  __shared__ uint32_t lut[VALUES ? 256 : 1];
  for (int i = threadIdx.x; i < 512; i += kThreads) {
    uint32_t e, c;
    bp8_qentry_signed(i, NEAREST, e, c);
    tbl[i] = make_uint2(e, c);
  }
  if (VALUES) lut[threadIdx.x] = threadIdx.x == 0x80 ? 0x7FC00000u : posit_to_f32_bits<8, 2>(threadIdx.x);
  __syncthreads();
  auto enc = [&](uint32_t u) {
    const uint2 t = tbl[u >> 23];
    return bp8_encode_signed(u, t.x, t.y);
  };
  const size_t nq = vec ? n / 4 : 0;
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
  uint32_t *cw = reinterpret_cast<uint32_t *>(codes);
  uint4 *v4 = reinterpret_cast<uint4 *>(vals);
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = blockIdx.x * tile; base < nq; base += (size_t)gridDim.x * tile) {
    uint4 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      v[j] = i < nq ? __ldcs(x4 + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      if (i < nq) {
        const uint32_t c0 = enc(v[j].x), c1 = enc(v[j].y), c2 = enc(v[j].z), c3 = enc(v[j].w);
        __stcs(cw + i, c0 | (c1 << 8) | (c2 << 16) | (c3 << 24));
        if (VALUES) __stcs(v4 + i, make_uint4(lut[c0], lut[c1], lut[c2], lut[c3]));
      }
    }
  }
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = nq * 4 + tid; i < n; i += stride) {
    const uint32_t c = enc(__float_as_uint(x[i]));
    codes[i] = (uint8_t)c;
    if (VALUES) vals[i] = __uint_as_float(lut[c]);
  }
}

// ------------------------------------------------------------ encode bp16 ---
// Signed per-binade table (bp16_qentry_signed, 512 entries): a code is one
// table load, the RTNE parity bit, a shift-add and a conditional negate
// (bp16_encode_signed).  Units of four elements (a float4 in, 8 bytes of codes
// out) in the decode kernels' tile order; grid-stride over tiles, 8 blocks per SM.
template <bool RTNE, int U>
__global__ void __launch_bounds__(kThreads) k_encode_bp16(const float *__restrict__ x, size_t n,
                                                          uint16_t *__restrict__ codes, bool vec) {
  __shared__ uint2 tbl[512];
  for (int i = threadIdx.x; i < 512; i += kThreads) {
    uint32_t e, c;
    bp16_qentry_signed(i, RTNE, e, c);
    tbl[i] = make_uint2(e, c);
  }
  __syncthreads();
  auto enc = [&](uint32_t u) {
    const uint2 t = tbl[u >> 23];
    return bp16_encode_signed<RTNE>(u, t.x, t.y);
  };
  const size_t nq = vec ? n / 4 : 0;
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
  uint2 *c2 = reinterpret_cast<uint2 *>(codes);
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = blockIdx.x * tile; base < nq; base += (size_t)gridDim.x * tile) {
    uint4 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      v[j] = i < nq ? __ldcs(x4 + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const size_t i = base + threadIdx.x + j * kThreads;
      if (i < nq)
        __stcs(c2 + i, make_uint2(enc(v[j].x) | (enc(v[j].y) << 16), enc(v[j].z) | (enc(v[j].w) << 16)));
    }
  }
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = nq * 4 + tid; i < n; i += stride) codes[i] = (uint16_t)enc(__float_as_uint(x[i]));
}

// ------------------------------------------------- grouped quantize (bp8) ---
// One warp per (row, group).  The exponent of the scaled value x / 2^s is
// formed as an integer (no rounding, no underflow), then the quantize table
// is applied to it.
__device__ __forceinline__ int ceil_log2_f32(uint32_t a) {   // a = |x| bits, a != 0
  int b = (int)(a >> 23);
  uint32_t M = a & 0x7FFFFFu;
  if (b == 0) {                         // subnormal: a = M * 2^-149
    int msb = 31 - __clz((int)M);
    return -149 + msb + ((M & (M - 1u)) ? 1 : 0);
  }
  return (b - 127) + (M ? 1 : 0);
}

__device__ __forceinline__ uint32_t q8_scaled(const uint2 *tbl, uint32_t u, int s) {
  uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x80u;
  if (a == 0u) return 0u;
  int b = (int)(a >> 23);
  uint32_t M = a & 0x7FFFFFu;
  int E;
  if (b == 0) {                         // normalise a subnormal input
    int msb = 31 - __clz((int)M);
    E = -149 + msb;
    M = (M << (23 - msb)) & 0x7FFFFFu;
  } else if (b == 255) {
    E = 1000;                           // inf: saturates
  } else {
    E = b - 127;
  }
  int be = E - s + 127;
  be = be < 1 ? 1 : (be > 255 ? 255 : be);
  uint2 t = tbl[be];
  QEntry q{t.x, t.y};
  uint32_t mag = bp8_apply(q, M);
  return (u >> 31) ? ((0u - mag) & 0xFFu) : mag;
}

template <bool NEAREST>
__global__ void __launch_bounds__(kThreads) k_group_quantize_bp8(const float *__restrict__ x, int rows,
                                                                 int K, int group, int G,
                                                                 bool compute, int maxpos_log2,
                                                                 int32_t *__restrict__ exps,
                                                                 uint8_t *__restrict__ codes) {
  __shared__ uint2 tbl[256];
  {
    QEntry q = bp8_qentry(threadIdx.x, NEAREST);
    tbl[threadIdx.x] = make_uint2(q.lo_sh, q.thr);
  }
  __syncthreads();
  int lane = threadIdx.x & 31;
  long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  long long total = (long long)rows * G;
  for (long long w = warp; w < total; w += nwarps) {
    int r = (int)(w / G), g = (int)(w % G);
    int k0 = g * group, k1 = min(K, k0 + group);
    const float *row = x + (size_t)r * K;
    int s;
    if (compute) {
      uint32_t amax = 0u;
      for (int k = k0 + lane; k < k1; k += 32) {
        uint32_t a = __float_as_uint(row[k]) & 0x7FFFFFFFu;
        if (a > 0x7F800000u) a = 0u;          // NaN does not take part in absmax
        amax = max(amax, a);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      s = amax ? (amax >= 0x7F800000u ? 128 - maxpos_log2 : ceil_log2_f32(amax) - maxpos_log2) : 0;
      if (lane == 0) exps[w] = s;
    } else {
      s = exps[w];
    }
    for (int k = k0 + lane; k < k1; k += 32)
      codes[(size_t)r * K + k] = (uint8_t)q8_scaled(tbl, __float_as_uint(row[k]), s);
  }
}

// ------------------------------------------------------------- quire->bp32 ---
template <int NL>
__global__ void __launch_bounds__(kThreads) k_quire_to_bp32(const uint32_t *__restrict__ limbs, size_t n,
                                                            uint32_t *__restrict__ out) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    uint32_t q[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) q[j] = limbs[i * NL + j];
    out[i] = bp32_from_limbs<NL>(q);
  }
}

// quire256_to_bposit16 of [n, NL] limbs: the bp16 prefix of the bposit32
// round (bp16_from_bp32).
template <int NL>
__global__ void __launch_bounds__(kThreads) k_quire_to_bp16(const uint32_t *__restrict__ limbs, size_t n,
                                                            uint16_t *__restrict__ out) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    uint32_t q[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) q[j] = limbs[i * NL + j];
    out[i] = bp16_from_bp32(bp32_from_limbs<NL>(q));
  }
}

__global__ void __launch_bounds__(kThreads) k_bp32_to_bp16(const uint32_t *__restrict__ codes, size_t n,
                                                           uint16_t *__restrict__ out) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) out[i] = bp16_from_bp32(codes[i]);
}

}  // namespace

// --------------------------------------------------------------- launchers ---
// One block per tile of kThreads * U units of `per` elements (at least one block).
inline int tile_grid(size_t n, int per, int U) {
  const size_t tile = (size_t)kThreads * U * per;
  const size_t b = (n + tile - 1) / tile;
  return (int)std::min<size_t>(std::max<size_t>(b, 1), (size_t)1 << 30);
}

constexpr int kDecU8 = 4, kDecU16 = 8, kEncU16 = 8, kEncU8 = 8;

int launch_decode(int fmt, const void *codes, size_t n, float *out, cudaStream_t s) {
  if (n == 0) return kOk;
  const bool oal = aligned16(out);
  if (fmt == 8) {
    const bool vec = oal && ((uintptr_t)codes & 3u) == 0u;
    k_decode_bp8<kDecU8><<<tile_grid(n, 4, kDecU8), kThreads, 0, s>>>((const uint8_t *)codes, n, out, vec);
  } else {
    const bool vec = oal && ((uintptr_t)codes & 7u) == 0u;
    static bool attr_set[128] = {};   // per device: the 128 KB table needs the opt-in
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 128 && !attr_set[dev]) {
      if (cudaFuncSetAttribute(k_decode_bp16<kDecU16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kDec16Smem) != cudaSuccess)
        return set_error(kECuda, "decode: shared-memory opt-in: %s", cudaGetErrorString(cudaGetLastError()));
      attr_set[dev] = true;
    }
    const size_t tile = (size_t)kDec16Threads * kDecU16 * 4;
    const int g = (int)std::min<size_t>(std::max<size_t>((n + tile - 1) / tile, 1), (size_t)sm_count());
    k_decode_bp16<kDecU16><<<g, kDec16Threads, kDec16Smem, s>>>((const uint16_t *)codes, n, out, vec);
  }
  return check_launch("decode");
}

int launch_quantize_bp8(const float *x, size_t n, bool nearest, uint8_t *codes, float *values,
                        cudaStream_t s) {
  if (n == 0) return kOk;
  const bool vec = aligned16(x) && ((uintptr_t)codes & 3u) == 0u && (values == nullptr || aligned16(values));
  const int g = std::min(tile_grid(n, 4, kEncU8), sm_count() * 8);
  if (nearest) {
    if (values) k_quantize_bp8<true, true, kEncU8><<<g, kThreads, 0, s>>>(x, n, codes, values, vec);
    else k_quantize_bp8<true, false, kEncU8><<<g, kThreads, 0, s>>>(x, n, codes, values, vec);
  } else {
    if (values) k_quantize_bp8<false, true, kEncU8><<<g, kThreads, 0, s>>>(x, n, codes, values, vec);
    else k_quantize_bp8<false, false, kEncU8><<<g, kThreads, 0, s>>>(x, n, codes, values, vec);
  }
  return check_launch("quantize_bp8");
}

int launch_encode_bp16(const float *x, size_t n, bool rtne, uint16_t *codes, cudaStream_t s) {
  if (n == 0) return kOk;
  const bool vec = aligned16(x) && ((uintptr_t)codes & 7u) == 0u;
  const int g = std::min(tile_grid(n, 4, kEncU16), sm_count() * 8);
  if (rtne) k_encode_bp16<true, kEncU16><<<g, kThreads, 0, s>>>(x, n, codes, vec);
  else k_encode_bp16<false, kEncU16><<<g, kThreads, 0, s>>>(x, n, codes, vec);
  return check_launch("encode_bp16");
}

int launch_group_quantize_bp8(const float *x, int rows, int K, int group, bool nearest,
                              bool compute_scales, int maxpos_log2, int32_t *exps, uint8_t *codes,
                              cudaStream_t s) {
  if (rows == 0 || K == 0) return kOk;
  int G = (K + group - 1) / group;
  size_t warps = (size_t)rows * G;
  int g = grid_for(warps * 32);
  if (nearest)
    k_group_quantize_bp8<true><<<g, kThreads, 0, s>>>(x, rows, K, group, G, compute_scales, maxpos_log2, exps, codes);
  else
    k_group_quantize_bp8<false><<<g, kThreads, 0, s>>>(x, rows, K, group, G, compute_scales, maxpos_log2, exps, codes);
  return check_launch("group_quantize_bp8");
}

int launch_quire_to_bp16(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out, cudaStream_t s) {
  if (n == 0) return kOk;
  int g = grid_for(n);
  switch (nlimbs) {
    case 8: k_quire_to_bp16<8><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    case 12: k_quire_to_bp16<12><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    case 16: k_quire_to_bp16<16><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    default: return set_error(kEInval, "quire_to_bp16: nlimbs must be 8, 12 or 16 (got %d)", nlimbs);
  }
  return check_launch("quire_to_bp16");
}

int launch_bp32_to_bp16(const uint32_t *codes, size_t n, uint16_t *out, cudaStream_t s) {
  if (n == 0) return kOk;
  k_bp32_to_bp16<<<grid_for(n), kThreads, 0, s>>>(codes, n, out);
  return check_launch("bp32_to_bp16");
}

int launch_quire_to_bp32(const uint32_t *limbs, int nlimbs, size_t n, uint32_t *out, cudaStream_t s) {
  if (n == 0) return kOk;
  int g = grid_for(n);
  switch (nlimbs) {
    case 8: k_quire_to_bp32<8><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    case 12: k_quire_to_bp32<12><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    case 16: k_quire_to_bp32<16><<<g, kThreads, 0, s>>>(limbs, n, out); break;
    default: return set_error(kEInval, "quire_to_bp32: nlimbs must be 8, 12 or 16 (got %d)", nlimbs);
  }
  return check_launch("quire_to_bp32");
}

}  // namespace bp

// ------------------------------------------------------------ bp32 -> f64 ---
namespace bp {
namespace {

// value(bp32 code) * 2^(re[m] + ce[n]): rows over blocks, columns over threads.
__global__ void __launch_bounds__(256) k_bp32_to_f64(const uint32_t *__restrict__ codes, int M, int N,
                                                     const int32_t *__restrict__ re,
                                                     const int32_t *__restrict__ ce,
                                                     double *__restrict__ out) {
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    const int rex = re ? re[m] : 0;
    const size_t rb = (size_t)m * N;
    for (int n = threadIdx.x; n < N; n += blockDim.x)
      out[rb + n] = bp32_value_scaled(codes[rb + n], rex + (ce ? ce[n] : 0));
  }
}

// The same exact value (plus an optional fp32 column bias), rounded once to
// the nearest-even fp32 -- the hand-off to the next fp32 op of a model.  NaR,
// which no quire round produces but a GEMM that gave up on a bounded wait
// writes, becomes NaN here, so the failure shows in the model's output.
__global__ void __launch_bounds__(256) k_bp32_to_f32(const uint32_t *__restrict__ codes, int M, int N,
                                                     const int32_t *__restrict__ re,
                                                     const int32_t *__restrict__ ce,
                                                     const float *__restrict__ bias,
                                                     float *__restrict__ out) {
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    const int rex = re ? re[m] : 0;
    const size_t rb = (size_t)m * N;
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
      out[rb + n] = bp32_f32_out(codes[rb + n], rex + (ce ? ce[n] : 0), bias ? bias[n] : 0.0f);
    }
  }
}

}  // namespace

int launch_bp32_to_f32(const uint32_t *codes, int M, int N, const int32_t *re, const int32_t *ce,
                       const float *bias, float *out, cudaStream_t s) {
  if ((size_t)M * N == 0) return kOk;
  k_bp32_to_f32<<<std::min(M, sm_count() * 8), 256, 0, s>>>(codes, M, N, re, ce, bias, out);
  return check_launch("bp32_to_f32");
}

int launch_bp32_to_f64(const uint32_t *codes, int M, int N, const int32_t *re, const int32_t *ce,
                       double *out, cudaStream_t s) {
  if ((size_t)M * N == 0) return kOk;
  k_bp32_to_f64<<<std::min(M, sm_count() * 8), 256, 0, s>>>(codes, M, N, re, ce, out);
  return check_launch("bp32_to_f64");
}

}  // namespace bp

// ----------------------------------------------------- quantize bp8 (f64) ---
// The reference quantizes float64 (reference/bposit_fast.py:90); rounding
// such input to fp32 first could cross a midpoint, so this variant applies the
// same per-binade table to the 52-bit mantissa (shift + 29, threshold << 29).
namespace bp {
namespace {

template <bool NEAREST, bool VALUES>
__global__ void __launch_bounds__(256) k_quantize_bp8_f64(const unsigned long long *__restrict__ x, size_t n,
                                                          uint8_t *__restrict__ codes,
                                                          unsigned long long *__restrict__ vals) {
  __shared__ uint2 tbl[256];
  __shared__ uint32_t lut[256];
  {
    QEntry q = bp8_qentry(threadIdx.x, NEAREST);
    tbl[threadIdx.x] = make_uint2(q.lo_sh, q.thr);
    lut[threadIdx.x] = posit_to_f32_bits<8, 2>(threadIdx.x);
  }
  __syncthreads();
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    unsigned long long u = x[i];
    unsigned long long a = u & 0x7FFFFFFFFFFFFFFFull;
    uint32_t code;
    if (a > 0x7FF0000000000000ull) {
      code = 0x80u;
    } else {
      int b64 = (int)(a >> 52);
      unsigned long long M = a & 0xFFFFFFFFFFFFFull;
      int b32 = b64 == 0 ? 0 : (b64 - 1023 + 127);
      if (b64 != 0) b32 = b32 < 1 ? 1 : (b32 > 255 ? 255 : b32);
      uint2 t = tbl[b32];
      uint32_t sh = (t.x >> 8) + 29u;
      unsigned long long thr = t.y == 0x7FFFFFu ? 0xFFFFFFFFFFFFFull : ((unsigned long long)t.y << 29);
      unsigned long long mask = (1ull << sh) - 1ull;
      uint32_t mag = (t.x & 0xFFu) + (uint32_t)(M >> sh) + ((M & mask) > thr ? 1u : 0u);
      code = (u >> 63) ? ((0u - mag) & 0xFFu) : mag;
    }
    codes[i] = (uint8_t)code;
    if (VALUES) {
      unsigned long long v;
      if (code == 0x80u) v = 0x7FF8000000000000ull;
      else if (code == 0u) v = u & 0x8000000000000000ull;          // +-0 keeps its sign
      else v = __double_as_longlong((double)__uint_as_float(lut[code]));
      vals[i] = v;
    }
  }
}

}  // namespace

int launch_quantize_bp8_f64(const double *x, size_t n, bool nearest, uint8_t *codes, double *values,
                            cudaStream_t s) {
  if (n == 0) return kOk;
  size_t blocks = (n + 255) / 256, cap = (size_t)sm_count() * 8;
  int g = (int)(blocks < cap ? blocks : cap);
  auto xu = (const unsigned long long *)x;
  auto vu = (unsigned long long *)values;
  if (nearest) {
    if (values) k_quantize_bp8_f64<true, true><<<g, 256, 0, s>>>(xu, n, codes, vu);
    else k_quantize_bp8_f64<true, false><<<g, 256, 0, s>>>(xu, n, codes, vu);
  } else {
    if (values) k_quantize_bp8_f64<false, true><<<g, 256, 0, s>>>(xu, n, codes, vu);
    else k_quantize_bp8_f64<false, false><<<g, 256, 0, s>>>(xu, n, codes, vu);
  }
  return check_launch("quantize_bp8_f64");
}

}  // namespace bp
