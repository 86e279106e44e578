// bp_gemm.cu -- quire GEMM front end: per-row operand statistics, workspace
// layout and the choice between the tensor-core and CUDA-core paths.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_gemm_common.cuh"
#include "bp_internal.cuh"

namespace bp {

int launch_gemm_simt(const GemmArgs &a, int4 *sta, int4 *stb, cudaStream_t s);
int launch_gemm_tc(const GemmArgs &a, int4 *sta, int4 *stb, void *ws, size_t ws_bytes, int algo,
                   int a_mode, cudaStream_t s);
size_t gemm_tc_workspace(int fmt, int M, int N, int K, int algo);
bool gemm_tc_supported(int fmt, int M, int N, int K);

namespace {

// Per row of an operand: {lowest possible set-bit exponent, highest binade,
// any nonzero, 0}, over the row's elements with the group scale folded in.
// One warp per row.
template <int FMT>
__global__ void __launch_bounds__(256) k_row_stats(const void *__restrict__ codes, int rows, int K,
                                                   const int32_t *__restrict__ s, int G, int group,
                                                   int4 *__restrict__ stats, const void *__restrict__ codes2,
                                                   int rows2, const int32_t *__restrict__ s2,
                                                   int4 *__restrict__ stats2) {
  // rows [0, rows) of `codes` and then rows [0, rows2) of `codes2` (the other
  // operand, same K), one warp per row: both operands in one launch
  int lane = threadIdx.x & 31;
  long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long rr = warp; rr < (long long)rows + rows2; rr += nw) {
    const bool second = rr >= rows;
    const long long r = second ? rr - rows : rr;
    const void *cb = second ? codes2 : codes;
    const int32_t *sc = second ? s2 : s;
    int lo = 0x3FFFFFFF, hi = -0x3FFFFFFF, nz = 0;
    for (int k = lane; k < K; k += 32) {
      uint32_t c = FMT == 8 ? ((const uint8_t *)cb)[(size_t)r * K + k] : ((const uint16_t *)cb)[(size_t)r * K + k];
      Dec d = FMT == 8 ? decode_posit<8, 2>(c) : decode_posit<16, 3>(c);
      if (d.kind != 0) continue;
      int scl = sc ? sc[(size_t)r * G + k / group] : 0;
      lo = min(lo, d.scale - d.fw + scl);
      hi = max(hi, d.scale + scl);
      nz = 1;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
      nz |= __shfl_xor_sync(0xFFFFFFFFu, nz, o);
    }
    if (lane == 0) (second ? stats2 : stats)[r] = make_int4(nz ? lo : 0, nz ? hi : 0, nz, 0);
  }
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

int launch_row_stats2(int fmt, const void *codes, int rows, const int32_t *s, int4 *stats, const void *codes2,
                      int rows2, const int32_t *s2, int4 *stats2, int K, int group, cudaStream_t st) {
  if (rows + rows2 == 0) return kOk;
  int G = group > 0 ? (K + group - 1) / group : 1;
  long long blocks = (((long long)rows + rows2) * 32 + 255) / 256;
  long long cap = (long long)sm_count() * 8;
  int g = (int)(blocks < cap ? blocks : cap);
  if (g < 1) g = 1;
  const int gr = group > 0 ? group : 1;
  if (fmt == 8) k_row_stats<8><<<g, 256, 0, st>>>(codes, rows, K, s, G, gr, stats, codes2, rows2, s2, stats2);
  else k_row_stats<16><<<g, 256, 0, st>>>(codes, rows, K, s, G, gr, stats, codes2, rows2, s2, stats2);
  return check_launch("row_stats");
}

int launch_row_stats(int fmt, const void *codes, int rows, int K, const int32_t *s, int group,
                     int4 *stats, cudaStream_t st) {
  return launch_row_stats2(fmt, codes, rows, s, stats, nullptr, 0, nullptr, nullptr, K, group, st);
}

static size_t stats_bytes(int M, int N) { return align_up((size_t)(M + N) * sizeof(int4), 256); }

static bool use_tc(const GemmArgs &a, int algo) {
  if (algo == 1) return false;
  if (!gemm_tc_supported(a.fmt, a.M, a.N, a.K)) return false;
  if (algo >= 2) return true;
  // auto: tensor cores once there is enough work to fill the machine
  return (long long)a.M * a.N >= 128LL * 128 * 8 && a.K >= 64;
}

bool gemm_uses_tc(const GemmArgs &a, int algo) { return use_tc(a, algo); }

size_t gemm_workspace_size(int fmt, int M, int N, int K, int algo) {
  size_t ws = stats_bytes(M, N);
  if (algo != 1 && gemm_tc_supported(fmt, M, N, K)) ws += gemm_tc_workspace(fmt, M, N, K, algo);
  return ws;
}

int launch_quire_gemm(const GemmArgs &a, int algo, void *ws, size_t ws_bytes, cudaStream_t s, int a_mode) {
  size_t need_stats = stats_bytes(a.M, a.N);
  if (ws_bytes < need_stats) return set_error(kEWorkspace, "quire_gemm: workspace too small");
  int4 *sta = (int4 *)ws;
  int4 *stb = sta + a.M;
  if (use_tc(a, algo)) {   // the tensor-core prep computes the row statistics itself
    size_t need = gemm_tc_workspace(a.fmt, a.M, a.N, a.K, algo);
    if (ws_bytes < need_stats + need) return set_error(kEWorkspace, "quire_gemm: workspace too small");
    return launch_gemm_tc(a, sta, stb, (char *)ws + need_stats, ws_bytes - need_stats, algo, a_mode, s);
  }
  if (a_mode == 2 || a_mode == 3) return kOk;   // the CUDA-core path prepares nothing ahead
  int rc = launch_row_stats2(a.fmt, a.A, a.M, a.sa, sta, a.B, a.N, a.sb, stb, a.K, a.group, s);
  if (rc) return rc;
  return launch_gemm_simt(a, sta, stb, s);
}

}  // namespace bp
