// bp_w8a8.cu -- the activation side of the reference's W8A8 recipe in one
// kernel: per row, recommended_exponents (reference/bposit_quantize.py:46-63)
// and the truncating bp8 encode of the row scaled by 2^-e
// (encode_bposit8 on floats, reference/bposit_ref.py:258-270).
//
// One warp per row (rows of up to kStageK elements staged in the warp's slice
// of shared memory, longer ones re-read through L2), no block-wide barrier:
//   rms  = sqrt(sum(x^2) / K)                       float64, warp reduction
//   p95  = numpy's 'linear' percentile of |x| at 95: the order statistics at
//          ranks lo = floor(0.95 (K - 1)) and lo + 1 by a 4-pass radix select
//          on the fp32 bit patterns of |x| (their order is the values'), with
//          a 256-bin histogram per warp, then lerp exactly as numpy does
//          (b - (b - a)(1 - t) when t >= 0.5); skipped when a count of
//          |x| > 2 rms shows a[lo + 1] <= 2 rms (then ref = rms whatever p95 is)
//   ref  = p95 if p95 > 0 and p95 > 2 rms, else rms;  e = rint(log2(ref)),
//          0 for an all-zero row
//   code = truncating bp8 of x * 2^-e (exact in float64), 0 when
//          |x * 2^-e| <= the largest double below 1/(2 * 10^8)
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
constexpr int kStageK = 1024;   // rows up to this length are staged in shared memory

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ uint32_t warp_sum_u(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
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

template <bool STAGED>
__global__ void __launch_bounds__(kT) k_w8a8_rows(const float *__restrict__ x, int rows, int K,
                                                  int32_t *__restrict__ exps, uint8_t *__restrict__ codes) {
  __shared__ uint2 tbl[256];          // truncating bp8 quantize table (bp8_qentry)
  __shared__ uint32_t hists[kWarps][256];
  extern __shared__ float s_rows[];   // [kWarps][K] when STAGED
  {
    QEntry q = bp8_qentry(threadIdx.x, false);
    tbl[threadIdx.x] = make_uint2(q.lo_sh, q.thr);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t *hist = hists[warp];
  float *srow = STAGED ? s_rows + (size_t)warp * K : nullptr;
  const double pos = 0.95 * (double)(K - 1);
  const int lo = (int)floor(pos);
  const double t = pos - (double)lo;
  const int kpad = (K + 31) / 32 * 32;   // every lane runs every trip of the histogram loop
  for (int r = blockIdx.x * kWarps + warp; r < rows; r += gridDim.x * kWarps) {
    const float *xg = x + (size_t)r * K;
    double ss = 0.0;
    for (int k = lane; k < K; k += 32) {
      const float f = xg[k];
      if (STAGED) srow[k] = f;
      ss += (double)f * (double)f;
    }
    const double rms = sqrt(warp_sum_d(ss) / (double)K);
    __syncwarp();
    const float *xr = STAGED ? srow : xg;
    // The percentile only matters when it exceeds 2 rms.  With c = #{|x| > 2 rms}:
    // c <= K - lo - 2 means a[lo + 1] <= 2 rms, so p95 (between a[lo] and
    // a[lo + 1]) does not exceed it and ref = rms without the selection.
    uint32_t cnt = 0u;
    const double two_rms = 2.0 * rms;
    for (int k = lane; k < K; k += 32) cnt += fabs((double)xr[k]) > two_rms ? 1u : 0u;
    cnt = warp_sum_u(cnt);
    const bool need_p95 = rms > 0.0 && (long long)cnt > (long long)K - lo - 2;
    // radix select of rank lo among the keys |x| (fp32 bits, sign cleared)
    uint32_t prefix = 0u, mask = 0u, rank = (uint32_t)lo, eq = 0u;
    for (int shift = 24; shift >= 0 && need_p95; shift -= 8) {
#pragma unroll
      for (int q = 0; q < 8; ++q) hist[lane * 8 + q] = 0u;
      __syncwarp();
      for (int k = lane; k < kpad; k += 32) {
        const uint32_t key = k < K ? (__float_as_uint(xr[k]) & 0x7FFFFFFFu) : 0u;
        hist_add(hist, (key >> shift) & 255u, k < K && (key & mask) == prefix);
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
    const double a_lo = (double)__uint_as_float(prefix);
    // rank lo + 1: the same key while it repeats, else the next larger key
    double a_hi = a_lo;
    if (need_p95 && lo + 1 < K && rank + 1 >= eq) {
      uint32_t nxt = 0xFFFFFFFFu;
      for (int k = lane; k < K; k += 32) {
        const uint32_t key = __float_as_uint(xr[k]) & 0x7FFFFFFFu;
        if (key > prefix) nxt = min(nxt, key);
      }
      a_hi = (double)__uint_as_float(warp_min_u(nxt));
    }
    const double d = a_hi - a_lo;
    const double p95 = t >= 0.5 ? a_hi - d * (1.0 - t) : a_lo + d * t;
    int e = 0;
    if (rms > 0.0) {
      const double ref = (need_p95 && p95 > 0.0 && p95 > 2.0 * rms) ? p95 : rms;
      e = (int)rint(log2(ref));
    }
    if (lane == 0) exps[r] = e;
    // truncating encode of x * 2^-e (float64 bit logic of the bp8 f64 quantizer)
    const double sc = scalbn(1.0, -e);
    uint8_t *cr = codes + (size_t)r * K;
    for (int k = lane; k < K; k += 32) {
      const double v = (double)xr[k] * sc;
      const unsigned long long u = (unsigned long long)__double_as_longlong(v);
      const unsigned long long a = u & 0x7FFFFFFFFFFFFFFFull;
      uint32_t code;
      if (a > 0x7FF0000000000000ull) {
        code = 0x80u;
      } else if (__longlong_as_double((long long)a) <= BP_LIMIT_ZERO) {
        code = 0u;
      } else {
        const int b64 = (int)(a >> 52);
        const unsigned long long Mm = a & 0xFFFFFFFFFFFFFull;
        int b32 = b64 - 1023 + 127;
        b32 = b32 < 1 ? 1 : (b32 > 255 ? 255 : b32);
        const uint2 q = tbl[b32];
        const uint32_t sh = (q.x >> 8) + 29u;
        const unsigned long long thr = q.y == 0x7FFFFFu ? 0xFFFFFFFFFFFFFull : ((unsigned long long)q.y << 29);
        const unsigned long long msk = (1ull << sh) - 1ull;
        const uint32_t mag = (q.x & 0xFFu) + (uint32_t)(Mm >> sh) + ((Mm & msk) > thr ? 1u : 0u);
        code = (u >> 63) ? ((0u - mag) & 0xFFu) : mag;
      }
      cr[k] = (uint8_t)code;
    }
    __syncwarp();   // the next row reuses this warp's staging and histogram
  }
}

}  // namespace

int launch_w8a8_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, cudaStream_t s) {
  if (rows == 0 || K == 0) return kOk;
  const int blocks = (rows + kWarps - 1) / kWarps;
  if (K <= kStageK) {
    // 32 KB of staging at most: several blocks per SM stay resident
    const size_t smem = (size_t)kWarps * K * sizeof(float);
    k_w8a8_rows<true><<<std::min(blocks, sm_count() * 6), kT, smem, s>>>(x, rows, K, exps, codes);
  } else {
    // long rows through L2: 4 blocks (32 rows) per SM in flight keep the
    // re-read rows of a 4864-wide activation (~90 MB) inside L2
    k_w8a8_rows<false><<<std::min(blocks, sm_count() * 4), kT, 0, s>>>(x, rows, K, exps, codes);
  }
  return check_launch("w8a8_rows");
}

}  // namespace bp
