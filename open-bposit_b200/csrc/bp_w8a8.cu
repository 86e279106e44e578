// bp_w8a8.cu -- the activation side of the reference's W8A8 recipe in one
// kernel: per row, recommended_exponents (reference/bposit_quantize.py:46-63)
// and the truncating bp8 encode of the row scaled by 2^-e
// (encode_bposit8 on floats, reference/bposit_ref.py:258-270).
//
// One block per row (grid-stride over rows):
//   rms  = sqrt(sum(x^2) / K)                       float64, block reduction
//   p95  = numpy's 'linear' percentile of |x| at 95: the order statistics at
//          ranks lo = floor(0.95 (K - 1)) and lo + 1 by a 4-pass radix select
//          on the fp32 bit patterns of |x| (their order is the values'),
//          then lerp exactly as numpy does (b - (b - a)(1 - t) when t >= 0.5);
//          skipped when a count of |x| > 2 rms shows a[lo + 1] <= 2 rms
//          (then ref = rms whatever p95 is)
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

constexpr int kT = 256;

__device__ __forceinline__ double block_sum_d(double v, double *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
  for (int w = 0; w < kT / 32; ++w) r += red[w];
  return r;
}

__device__ __forceinline__ uint32_t block_min_u(uint32_t v, uint32_t *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = red[0];
  for (int w = 1; w < kT / 32; ++w) r = min(r, red[w]);
  return r;
}

// Histogram add with warp aggregation: lanes that hit the same bin add once
// (the exponent byte of |x| is shared by most of a row).
__device__ __forceinline__ void hist_add(uint32_t *hist, uint32_t bin, bool active) {
  const uint32_t act = __ballot_sync(0xFFFFFFFFu, active);
  if (!active) return;
  const uint32_t peers = __match_any_sync(act, bin);
  if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
}

// Rows of up to SMEM_K elements are staged in shared memory once; longer rows
// are re-read from global memory (L2) by every pass.
constexpr int SMEM_K = 10240;

__global__ void __launch_bounds__(kT) k_w8a8_rows(const float *__restrict__ x, int rows, int K,
                                                  int32_t *__restrict__ exps, uint8_t *__restrict__ codes) {
  __shared__ uint2 tbl[256];          // truncating bp8 quantize table (bp8_qentry)
  __shared__ uint32_t hist[256];
  __shared__ double redd[kT / 32];
  __shared__ uint32_t redu[kT / 32];
  __shared__ uint32_t s_prefix, s_rank, s_eq;
  extern __shared__ float s_row[];
  {
    QEntry q = bp8_qentry(threadIdx.x, false);
    tbl[threadIdx.x] = make_uint2(q.lo_sh, q.thr);
  }
  __syncthreads();
  const bool staged = K <= SMEM_K;
  const double pos = 0.95 * (double)(K - 1);
  const int lo = (int)floor(pos);
  const double t = pos - (double)lo;
  const int kpad = (K + kT - 1) / kT * kT;   // every lane runs every loop trip (warp collectives)
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xg = x + (size_t)r * K;
    double ss = 0.0;
    for (int k = threadIdx.x; k < K; k += kT) {
      const float f = xg[k];
      if (staged) s_row[k] = f;
      ss += (double)f * (double)f;
    }
    const double rms = sqrt(block_sum_d(ss, redd) / (double)K);   // (its syncs also publish s_row)
    const float *xr = staged ? s_row : xg;
    // The percentile only matters when it exceeds 2 rms.  With c = #{|x| > 2 rms}:
    // c <= K - lo - 2 means a[lo + 1] <= 2 rms, so p95 (between a[lo] and
    // a[lo + 1]) does not exceed it and ref = rms without the selection.
    uint32_t cnt = 0u;
    const double two_rms = 2.0 * rms;
    for (int k = threadIdx.x; k < K; k += kT) cnt += fabs((double)xr[k]) > two_rms ? 1u : 0u;
    cnt = (uint32_t)block_sum_d((double)cnt, redd);
    const bool need_p95 = rms > 0.0 && (long long)cnt > (long long)K - lo - 2;
    // radix select of rank lo among the keys |x| (fp32 bits, sign cleared)
    uint32_t prefix = 0u, mask = 0u, rank = (uint32_t)lo;
    for (int shift = 24; shift >= 0 && need_p95; shift -= 8) {
      hist[threadIdx.x] = 0u;
      __syncthreads();
      for (int k = threadIdx.x; k < kpad; k += kT) {
        const uint32_t key = k < K ? (__float_as_uint(xr[k]) & 0x7FFFFFFFu) : 0u;
        hist_add(hist, (key >> shift) & 255u, k < K && (key & mask) == prefix);
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // lane l owns bins 8l .. 8l+7: inclusive prefix over lanes, then the
        // first bin whose running count passes `rank`
        uint32_t c[8], tot = 0u;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c[q] = hist[8 * threadIdx.x + q];
          tot += c[q];
        }
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if ((int)threadIdx.x >= o) incl += y;
        }
        const uint32_t excl = incl - tot;
        const bool mine = excl <= rank && rank < incl;
        if (mine) {
          uint32_t below = excl, b = 8u * threadIdx.x;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (below + c[q] <= rank && q < 7) {
              below += c[q];
              ++b;
            } else {
              break;
            }
          s_prefix = prefix | (b << shift);
          s_rank = rank - below;
          s_eq = hist[b];
        }
      }
      __syncthreads();
      prefix = s_prefix;
      rank = s_rank;
      mask |= 255u << shift;
    }
    const double a_lo = (double)__uint_as_float(prefix);
    // rank lo + 1: the same key while it repeats, else the next larger key
    double a_hi = a_lo;
    if (need_p95 && lo + 1 < K && rank + 1 >= s_eq) {
      uint32_t nxt = 0xFFFFFFFFu;
      for (int k = threadIdx.x; k < K; k += kT) {
        const uint32_t key = __float_as_uint(xr[k]) & 0x7FFFFFFFu;
        if (key > prefix) nxt = min(nxt, key);
      }
      nxt = block_min_u(nxt, redu);
      a_hi = (double)__uint_as_float(nxt);
    }
    const double d = a_hi - a_lo;
    const double p95 = t >= 0.5 ? a_hi - d * (1.0 - t) : a_lo + d * t;
    int e = 0;
    if (rms > 0.0) {
      const double ref = (need_p95 && p95 > 0.0 && p95 > 2.0 * rms) ? p95 : rms;
      e = (int)rint(log2(ref));
    }
    if (threadIdx.x == 0) exps[r] = e;
    // truncating encode of x * 2^-e (float64 bit logic of the bp8 f64 quantizer)
    const double sc = scalbn(1.0, -e);
    uint8_t *cr = codes + (size_t)r * K;
    for (int k = threadIdx.x; k < K; k += kT) {
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
    __syncthreads();
  }
}

}  // namespace

int launch_w8a8_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, cudaStream_t s) {
  if (rows == 0 || K == 0) return kOk;
  const size_t smem = K <= SMEM_K ? (size_t)K * sizeof(float) : 0;
  k_w8a8_rows<<<std::min(rows, sm_count() * 4), kT, smem, s>>>(x, rows, K, exps, codes);
  return check_launch("w8a8_rows");
}

}  // namespace bp
