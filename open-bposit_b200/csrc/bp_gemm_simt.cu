// bp_gemm_simt.cu -- exact quire GEMM on CUDA cores, and the per-row operand
// statistics shared with the tensor-core path.
//
// out[m, n] = quire256_to_bposit32( sum_k trunc0( v(A[m,k]) * v(B[n,k]) *
//                                   2^(sa[m,k/group] + sb[n,k/group]) * 2^96 ) )
// which is dot_at_precision's per-term rule (reference/bposit_ref.py:1028-1035,
// bposit_fast.dot_quire / matmul_quire reference/bposit_fast.py:102-176) with an
// optional power-of-two group scale folded into each element's exponent.
//
// Every code is an exact integer form m * 2^e (|m| < 2^12).  Per row we know
// the lowest possible set bit (emin) and the highest binade (emax), so a whole
// dot product lives in a window of the quire that is usually far narrower
// than 256 bits.  When that window starts at or above the quire's bit 0 (no
// term needs truncation) and fits 127 bits with the K-term carry head-room,
// the output is accumulated exactly in one 128-bit register pair (fast path).
// Otherwise the thread falls back to a 512-bit quire in local memory with
// per-term truncation toward zero (slow path; never taken for bp8 without
// group scales).
//
// Work split: a block of 256 threads owns TM x TN outputs and every output is
// shared by KS adjacent lanes, lane ks taking the terms k = ks, ks + KS, ...
// of each staged K chunk; the KS exact 128-bit partial sums are added with
// warp shuffles (exact: every partial and the total lie in the same window).
// A 16 x 576 x 576 linear is then 144 blocks, one per SM, instead of 36.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_internal.cuh"
#include "bp_gemm_common.cuh"

namespace bp {
namespace {

constexpr int TM = 8, TN = 8, KS = 4, KC = 32;
static_assert(TM * TN * KS == 256 && (KS & (KS - 1)) == 0 && KS <= 32, "block shape");

template <int FMT>
__global__ void __launch_bounds__(TM *TN *KS) k_quire_gemm_simt(GemmArgs a, const int4 *__restrict__ sta,
                                                                 const int4 *__restrict__ stb) {
  __shared__ int sAm[TM][KC + 1], sAe[TM][KC + 1];
  __shared__ int sBm[TN][KC + 1], sBe[TN][KC + 1];
  const int ks = threadIdx.x % KS, o = threadIdx.x / KS;
  const int tx = o % TN, ty = o / TN;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int m = m0 + ty, n = n0 + tx;
  const bool valid = m < a.M && n < a.N;
  int4 ra = valid ? sta[m] : make_int4(0, 0, 0, 0);
  int4 rb = valid ? stb[n] : make_int4(0, 0, 0, 0);
  const bool nz = ra.z && rb.z;
  const int base = ra.x + rb.x + 96;   // quire bit of the lowest possible term bit
  const int width = fast_width(ra, rb, a.K, FMT);
  const bool fast = nz && base >= 0 && width <= 127;
  unsigned __int128 acc = 0;
  for (int k0 = 0; k0 < a.K; k0 += KC) {
    for (int t = threadIdx.x; t < (TM + TN) * KC; t += TM * TN * KS) {
      const bool isa = t < TM * KC;
      const int tt = isa ? t : t - TM * KC;
      const int r = tt / KC, kk = tt % KC, k = k0 + kk;
      ElemME x{0, 0};
      if (isa) {
        if (k < a.K && m0 + r < a.M) x = load_elem<FMT>(a.A, m0 + r, a.K, k, a.sa, a.G, a.group);
        sAm[r][kk] = x.m;
        sAe[r][kk] = x.e;
      } else {
        if (k < a.K && n0 + r < a.N) x = load_elem<FMT>(a.B, n0 + r, a.K, k, a.sb, a.G, a.group);
        sBm[r][kk] = x.m;
        sBe[r][kk] = x.e;
      }
    }
    __syncthreads();
    if (fast) {
      const int off = ra.x + rb.x;
#pragma unroll
      for (int kk = ks; kk < KC; kk += KS) {
        int P = sAm[ty][kk] * sBm[tx][kk];
        int sh = sAe[ty][kk] + sBe[tx][kk] - off;
        sh = min(max(sh, 0), 127);
        acc += (unsigned __int128)(__int128)(long long)P << sh;
      }
    }
    __syncthreads();
  }
  // add the KS partial sums of an output (adjacent lanes)
  unsigned long long lo = (unsigned long long)acc, hi = (unsigned long long)(acc >> 64);
#pragma unroll
  for (int d = 1; d < KS; d <<= 1) {
    const unsigned long long olo = __shfl_xor_sync(0xFFFFFFFFu, lo, d);
    const unsigned long long ohi = __shfl_xor_sync(0xFFFFFFFFu, hi, d);
    const unsigned long long s0 = lo + olo;
    hi = hi + ohi + (s0 < lo ? 1ull : 0ull);
    lo = s0;
  }
  acc = ((unsigned __int128)hi << 64) | lo;
  if (!valid || ks != 0) return;
  uint32_t *oq = a.quire ? a.quire + ((size_t)m * a.N + n) * a.nlimbs : nullptr;
  uint32_t code = 0u;
  if (!nz) {
    if (oq)
      for (int i = 0; i < a.nlimbs; ++i) oq[i] = 0u;
  } else if (fast) {
    code = write_fast_output(acc, base, nullptr, oq, a.nlimbs);
  } else {
    slow_output<FMT>(a, m, n, &code, oq);
  }
  store_output(a, m, n, code);
}

}  // namespace

int launch_gemm_simt(const GemmArgs &a, int4 *sta, int4 *stb, cudaStream_t s) {
  dim3 grid((a.N + TN - 1) / TN, (a.M + TM - 1) / TM);
  if (grid.y > 65535u) return set_error(kERange, "quire_gemm: M too large for the CUDA-core path");
  if (a.fmt == 8) k_quire_gemm_simt<8><<<grid, TM * TN * KS, 0, s>>>(a, sta, stb);
  else k_quire_gemm_simt<16><<<grid, TM * TN * KS, 0, s>>>(a, sta, stb);
  return check_launch("quire_gemm_simt");
}

}  // namespace bp
