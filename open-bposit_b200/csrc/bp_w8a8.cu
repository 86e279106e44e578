// bp_w8a8.cu -- the activation side of the reference's W8A8 recipe in one
// kernel: per row, recommended_exponents (reference/bposit_quantize.py:46-63)
// and the truncating bp8 encode of the row scaled by 2^-e
// (encode_bposit8 on floats, reference/bposit_ref.py:258-270).
//
// One warp per row (rows up to ~1800 elements staged in the warp's slice of
// shared memory, at least 4 warps per block; longer rows read through L2 by
// each pass), no block-wide barrier, float4 loads eight at a time per lane:
//   rms  = sqrt(sum(x^2) / K)                       float64, warp reduction
//   p95  = numpy's 'linear' percentile of |x| at 95: the order statistics at
//          ranks lo = floor(0.95 (K - 1)) and lo + 1 by a 4-pass radix select
//          on the fp32 bit patterns of |x| (their order is the values'), with
//          a 256-bin histogram per warp, over a list of the candidates
//          |x| > 2 rms only (at most K / 4 by Chebyshev; when the percentile
//          can matter its ranks are among them or just below), then lerp
//          exactly as numpy does (b - (b - a)(1 - t) when t >= 0.5); skipped
//          when the count of candidates shows a[lo + 1] <= 2 rms (then ref =
//          rms whatever p95 is).  Comparisons are integer compares of fp32
//          bit patterns (the round-down of 2 rms stands for it exactly)
//   ref  = p95 if p95 > 0 and p95 > 2 rms, else rms;  e = rint(log2(ref)),
//          0 for an all-zero row
//   code = truncating bp8 of x * 2^-e (integer exponent arithmetic on the fp32
//          bits), 0 when |x * 2^-e| <= the largest double below 1/(2 * 10^8)
// The only difference from the numpy rule is the order of the float64 sum of
// squares, which matters only when ref falls within an ulp of 2^(k + 1/2) or
// p95 within an ulp of 2 rms.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "bp_format.cuh"
#include "bp_internal.cuh"

namespace bp {
namespace {

constexpr int kT = 256, kWarps = kT / 32;
// 36 KB of staged rows and candidate lists per block: with the 10 KB of static
// tables and histograms the block stays within the 48 KB a launch gets without
// opt-in
constexpr size_t kStageBytes = 36 * 1024;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ uint32_t warp_max_u(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t warp_min_u(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Histogram add with lane aggregation: lanes that hit the same bin add once
// (the exponent byte of |x| is shared by most of a row).  Whole warp.
__device__ __forceinline__ void hist_add(uint32_t *hist, uint32_t bin, bool active) {
  const uint32_t act = __ballot_sync(0xFFFFFFFFu, active);
  if (!active) return;
  const uint32_t peers = __match_any_sync(act, bin);
  if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
}


// Shared-memory slice of one warp, in 4-byte words, rounded to 16-byte units:
// the staged row (K floats) and the candidate list (K / 4 + 1 keys).
__host__ __device__ __forceinline__ int w8a8_row_floats(int K) { return (K + 3) & ~3; }
__host__ __device__ __forceinline__ int w8a8_list_words(int K) { return (K / 4 + 1 + 3) & ~3; }

// Truncating bp8 code of x * 2^-e from the fp32 bits of x, with integer
// exponent arithmetic: the scaled value's biased exponent E - e + 127
// (clamped to the table's [1, 255], which saturates or flushes exactly as the
// table does for out-of-range binades) selects the per-binade truncating
// entry and the 23-bit mantissa is applied to it.  zkey: the fp32 bit pattern
// of the largest float <= the zero cut * 2^e; |x| at or below it gives 0 (the
// float entry's limit_denominator cut).  Identical to quantizing the exact
// float64 x * 2^-e.
__device__ __forceinline__ uint32_t w8a8_code(const uint2 *tbl, uint32_t u, int e, uint32_t zkey) {
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x80u;   // NaN -> NaR
  if (a <= zkey) return 0u;
  int E;
  uint32_t M = a & 0x7FFFFFu;
  const int b = (int)(a >> 23);
  if (b == 0) {                          // subnormal input: normalise
    const int msb = 31 - __clz((int)M);
    E = -149 + msb;
    M = (M << (23 - msb)) & 0x7FFFFFu;
  } else if (b == 255) {
    E = 1000;                            // inf: saturates
  } else {
    E = b - 127;
  }
  int be = E - e + 127;
  be = be < 1 ? 1 : (be > 255 ? 255 : be);
  const uint2 t = tbl[be];
  const QEntry q{t.x, t.y};
  const uint32_t mag = bp8_apply(q, M);
  return (u >> 31) ? ((0u - mag) & 0xFFu) : mag;
}

// One warp per row; blockDim.x / 32 warps per block, each with a K-float
// slice of the dynamic shared memory for the row (STAGED) followed by a
// K/4-entry candidate list, and a 256-bin histogram.  VEC: K % 4 == 0 and
// 16-byte aligned rows -- float4 loads, eight at a time in flight per lane,
// and four codes per 32-bit store.
template <bool STAGED, bool VEC>
__global__ void __launch_bounds__(kT) k_w8a8_rows(const float *__restrict__ x, int rows, int K,
                                                  int32_t *__restrict__ exps, uint8_t *__restrict__ codes) {
  __shared__ uint2 tbl[256];          // truncating bp8 quantize table (bp8_qentry)
  __shared__ uint32_t hists[kWarps][256];
  extern __shared__ __align__(16) float s_rows[];   // per warp: [K] row (STAGED), [K / 4 + 1] candidate keys
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    QEntry q = bp8_qentry(i, false);
    tbl[i] = make_uint2(q.lo_sh, q.thr);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  uint32_t *hist = hists[warp];
  // per warp: the row, then the candidate list, each a whole number of
  // 16-byte units so that every warp's row is float4-aligned
  const size_t rowf = STAGED ? (size_t)w8a8_row_floats(K) : 0, per_warp = rowf + (size_t)w8a8_list_words(K);
  float *srow = STAGED ? s_rows + (size_t)warp * per_warp : nullptr;
  uint32_t *cand = reinterpret_cast<uint32_t *>(s_rows + (size_t)warp * per_warp + rowf);
  const double pos = 0.95 * (double)(K - 1);
  const int lo = (int)floor(pos);
  const double t = pos - (double)lo;
  const int kpad = (K + 31) / 32 * 32;   // every lane runs every trip of the warp-collective loops
  const int K4 = K / 4;
  for (int r = blockIdx.x * nwarps + warp; r < rows; r += gridDim.x * nwarps) {
    const float *xg = x + (size_t)r * K;
    double ss = 0.0;
    if (VEC) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xg);
      float4 *s4 = reinterpret_cast<float4 *>(srow);
      for (int u0 = lane; u0 < K4; u0 += 256) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = u0 + 32 * j < K4 ? __ldcs(x4 + u0 + 32 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (STAGED && u0 + 32 * j < K4) s4[u0 + 32 * j] = v[j];
          ss += (double)v[j].x * v[j].x + (double)v[j].y * v[j].y + (double)v[j].z * v[j].z + (double)v[j].w * v[j].w;
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
        const float f = xg[k];
        if (STAGED) srow[k] = f;
        ss += (double)f * (double)f;
      }
    }
    const double rms = sqrt(warp_sum_d(ss) / (double)K);
    __syncwarp();
    const float *xr = STAGED ? srow : xg;
    // Candidates: |x| > 2 rms, in integers -- for fp32 |x| that is its bit
    // pattern above that of the largest float <= 2 rms.  By Chebyshev there
    // are at most K / 4 of them.  One pass counts and lists them and keeps the
    // largest non-candidate and the smallest candidate.
    const double two_rms = 2.0 * rms;
    const uint32_t tkey = __float_as_uint(__double2float_rd(two_rms)) & 0x7FFFFFFFu;
    uint32_t cnt = 0u, mx_non = 0u, mn_cand = 0xFFFFFFFFu;
    auto take = [&](uint32_t key, bool valid) {   // whole warp
      const bool c = valid && key > tkey;
      const uint32_t bal = __ballot_sync(0xFFFFFFFFu, c);
      if (c) {
        const uint32_t at = cnt + __popc(bal & lt_mask);
        if (at <= (uint32_t)(K / 4)) cand[at] = key;   // always: Chebyshev bounds the count by K / 4
        mn_cand = min(mn_cand, key);
      } else if (valid) {
        mx_non = max(mx_non, key);
      }
      cnt += __popc(bal);
    };
    if (VEC) {
      // eight float4 per lane in flight, then their 32 keys (the list's order is free)
      const uint4 *r4 = reinterpret_cast<const uint4 *>(xr);
      for (int u0 = 0; u0 < K4; u0 += 256) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int u = u0 + 32 * j + lane;
          v[j] = u < K4 ? r4[u] : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (u0 + 32 * j >= K4) break;   // warp-uniform
          const bool ok = u0 + 32 * j + lane < K4;
          take(v[j].x & 0x7FFFFFFFu, ok);
          take(v[j].y & 0x7FFFFFFFu, ok);
          take(v[j].z & 0x7FFFFFFFu, ok);
          take(v[j].w & 0x7FFFFFFFu, ok);
        }
      }
    } else {
      for (int k = lane; k < kpad; k += 32) take(k < K ? (__float_as_uint(xr[k]) & 0x7FFFFFFFu) : 0u, k < K);
    }
    __syncwarp();
    // The percentile only matters when it exceeds 2 rms: c <= K - lo - 2 means
    // a[lo + 1] <= 2 rms, so p95 (between a[lo] and a[lo + 1]) does not exceed
    // it and ref = rms without the selection.
    const bool need_p95 = rms > 0.0 && (long long)cnt > (long long)K - lo - 2;
    double a_lo = 0.0, a_hi = 0.0;
    if (need_p95 && lo < K - (int)cnt) {
      // lo = K - c - 1: a[lo] is the largest non-candidate, a[lo + 1] the smallest candidate
      a_lo = (double)__uint_as_float(warp_max_u(mx_non));
      a_hi = lo + 1 < K ? (double)__uint_as_float(warp_min_u(mn_cand)) : a_lo;
    } else if (need_p95) {
      // radix select of rank lo - (K - c) among the candidate keys (fp32 bits
      // of |x|; their order is the values')
      uint32_t prefix = 0u, mask = 0u, rank = (uint32_t)(lo - (K - (int)cnt)), eq = 0u;
      const int cpad = ((int)cnt + 31) / 32 * 32;
      for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
        for (int q = 0; q < 8; ++q) hist[lane * 8 + q] = 0u;
        __syncwarp();
        for (int i = lane; i < cpad; i += 32) {
          const uint32_t key = i < (int)cnt ? cand[i] : 0u;
          hist_add(hist, (key >> shift) & 255u, i < (int)cnt && (key & mask) == prefix);
        }
        __syncwarp();
        // lane l owns bins 8l .. 8l+7: inclusive prefix over lanes, then the
        // first bin whose running count passes `rank`
        uint32_t c[8], tot = 0u;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c[q] = hist[8 * lane + q];
          tot += c[q];
        }
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - tot;
        const bool mine = excl <= rank && rank < incl;
        uint32_t below = excl, b = 8u * lane, cb = c[0];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          cb = c[q];
          if (below + c[q] <= rank && q < 7) {
            below += c[q];
            ++b;
          } else {
            break;
          }
        }
        const int owner = __ffs(__ballot_sync(0xFFFFFFFFu, mine)) - 1;
        b = __shfl_sync(0xFFFFFFFFu, b, owner);
        below = __shfl_sync(0xFFFFFFFFu, below, owner);
        eq = __shfl_sync(0xFFFFFFFFu, cb, owner);
        prefix |= b << shift;
        rank -= below;
        mask |= 255u << shift;
        __syncwarp();
      }
      a_lo = (double)__uint_as_float(prefix);
      // rank lo + 1: the same key while it repeats, else the next larger key
      // (every key above a candidate's is a candidate's)
      a_hi = a_lo;
      if (lo + 1 < K && rank + 1 >= eq) {
        uint32_t nxt = 0xFFFFFFFFu;
        for (int i = lane; i < (int)cnt; i += 32)
          if (cand[i] > prefix) nxt = min(nxt, cand[i]);
        a_hi = (double)__uint_as_float(warp_min_u(nxt));
      }
    }
    const double d = a_hi - a_lo;
    const double p95 = t >= 0.5 ? a_hi - d * (1.0 - t) : a_lo + d * t;
    int e = 0;
    if (rms > 0.0) {
      const double ref = (need_p95 && p95 > 0.0 && p95 > 2.0 * rms) ? p95 : rms;
      e = (int)rint(log2(ref));
    }
    if (lane == 0) exps[r] = e;
    // truncating encode of x * 2^-e
    const uint32_t zkey = __float_as_uint(__double2float_rd(scalbn(BP_LIMIT_ZERO, e))) & 0x7FFFFFFFu;
    uint8_t *cr = codes + (size_t)r * K;
    if (VEC) {
      const uint4 *r4 = reinterpret_cast<const uint4 *>(xr);
      uint32_t *cw = reinterpret_cast<uint32_t *>(cr);
      for (int u0 = lane; u0 < K4; u0 += 256) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = u0 + 32 * j < K4 ? r4[u0 + 32 * j] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (u0 + 32 * j < K4)
            cw[u0 + 32 * j] = w8a8_code(tbl, v[j].x, e, zkey) | (w8a8_code(tbl, v[j].y, e, zkey) << 8) |
                              (w8a8_code(tbl, v[j].z, e, zkey) << 16) | (w8a8_code(tbl, v[j].w, e, zkey) << 24);
      }
    } else {
      for (int k = lane; k < K; k += 32) cr[k] = (uint8_t)w8a8_code(tbl, __float_as_uint(xr[k]), e, zkey);
    }
    __syncwarp();   // the next row reuses this warp's staging, list and histogram
  }
}

}  // namespace

int launch_w8a8_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, cudaStream_t s) {
  if (rows == 0 || K == 0) return kOk;
  const bool vec = (K % 4) == 0 && ((uintptr_t)x & 15u) == 0 && ((uintptr_t)codes & 3u) == 0;
  const size_t list = (size_t)w8a8_list_words(K) * sizeof(uint32_t);   // candidate list per warp
  const size_t staged = (size_t)w8a8_row_floats(K) * sizeof(float) + list;
  if (staged <= kStageBytes / 4) {   // at least 4 warps per block with staged rows
    // rows staged in shared memory: as many warps per block as the budget allows
    const int w = std::max(1, std::min(kWarps, (int)(kStageBytes / staged)));
    const int blocks = std::min((rows + w - 1) / w, sm_count() * 16);
    if (vec) k_w8a8_rows<true, true><<<blocks, 32 * w, w * staged, s>>>(x, rows, K, exps, codes);
    else k_w8a8_rows<true, false><<<blocks, 32 * w, w * staged, s>>>(x, rows, K, exps, codes);
  } else {
    // longer rows are read through L2 by each pass (only the candidate lists in
    // shared memory, so more warps per SM): ~7 warps per block for K = 4864
    const int w = std::max(1, std::min(kWarps, (int)(kStageBytes / list)));
    if (list > kStageBytes) return set_error(kERange, "w8a8_rows: rows of %d elements are too long", K);
    const int blocks = std::min((rows + w - 1) / w, sm_count() * 4);
    if (vec) k_w8a8_rows<false, true><<<blocks, 32 * w, w * list, s>>>(x, rows, K, exps, codes);
    else k_w8a8_rows<false, false><<<blocks, 32 * w, w * list, s>>>(x, rows, K, exps, codes);
  }
  return check_launch("w8a8_rows");
}

}  // namespace bp
