// bp_abi.cu -- the extern "C" entry points declared in include/bposit_b200.h:
// argument checks, error reporting, workspace handling and dispatch to the
// kernels.  No exception crosses this boundary.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <string.h>
#include <stdio.h>

#include <atomic>

#include "../../include/bposit_b200.h"
#include "bp_internal.cuh"

namespace bp {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<unsigned long long> g_launches{0};

int check_launch(const char *what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kECuda, "%s: %s", what, cudaGetErrorString(e));
  return kOk;
}

static std::atomic<int> g_sms[128];

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  int v = g_sms[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// 1 when the current device is compute capability 10.x (B200 / sm_100).
static std::atomic<int> g_ok[128];

void clear_error() { g_err[0] = 0; }

int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(kENoDev, "no CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(kENoDev, "device index %d out of range", dev);
  int v = g_ok[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return set_error(kENoDev, "cannot query device %d", dev);
    v = major == 10 ? 1 : -1;
    g_ok[dev].store(v, std::memory_order_relaxed);
  }
  if (v < 0) return set_error(kENoDev, "device %d is not an sm_100 (B200) GPU", dev);
  return kOk;
}

int tc_device_error(int *out);
int launch_bp32_to_f64(const uint32_t *codes, int M, int N, const int32_t *re, const int32_t *ce,
                       double *out, cudaStream_t s);

}  // namespace bp

using namespace bp;

#define BP_VERSION 100  // 0.1.0

#define TRY(x)            \
  do {                    \
    int _rc = (x);        \
    if (_rc != kOk) return _rc; \
  } while (0)

extern "C" {

int bp_version(void) { return BP_VERSION; }

const char *bp_last_error(void) { return g_err; }

unsigned long long bp_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int bp_device_error(int *out) {
  g_err[0] = 0;
  if (!out) return set_error(kEInval, "bp_device_error: null pointer");
  TRY(check_device());
  return tc_device_error(out);
}

int bp_decode(int fmt, const void *codes, size_t n, float *out, void *stream) {
  g_err[0] = 0;
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_decode: fmt must be 8 or 16 (got %d)", fmt);
  if (n && (!codes || !out)) return set_error(kEInval, "bp_decode: null pointer");
  TRY(check_device());
  return launch_decode(fmt, codes, n, out, (cudaStream_t)stream);
}

int bp_quantize_bp8(const float *x, size_t n, int nearest, uint8_t *codes, float *values, void *stream) {
  g_err[0] = 0;
  if (n && (!x || !codes)) return set_error(kEInval, "bp_quantize_bp8: null pointer");
  TRY(check_device());
  return launch_quantize_bp8(x, n, nearest != 0, codes, values, (cudaStream_t)stream);
}

int bp_quantize_bp8_f64(const double *x, size_t n, int nearest, uint8_t *codes, double *values, void *stream) {
  g_err[0] = 0;
  if (n && (!x || !codes)) return set_error(kEInval, "bp_quantize_bp8_f64: null pointer");
  TRY(check_device());
  return launch_quantize_bp8_f64(x, n, nearest != 0, codes, values, (cudaStream_t)stream);
}

int bp_quantize_bp8_grouped(const float *x, int rows, int K, int group, int nearest, int compute_scales,
                            int maxpos_log2, int32_t *exps, uint8_t *codes, void *stream) {
  g_err[0] = 0;
  if (rows < 0 || K < 0) return set_error(kEInval, "bp_quantize_bp8_grouped: negative size");
  if (group <= 0) return set_error(kEInval, "bp_quantize_bp8_grouped: group must be > 0");
  if ((size_t)rows * K != 0 && (!x || !codes || !exps)) return set_error(kEInval, "bp_quantize_bp8_grouped: null pointer");
  TRY(check_device());
  return launch_group_quantize_bp8(x, rows, K, group, nearest != 0, compute_scales != 0, maxpos_log2, exps,
                                   codes, (cudaStream_t)stream);
}

int bp_encode_bp16(const float *x, size_t n, int rtne, uint16_t *codes, void *stream) {
  g_err[0] = 0;
  if (n && (!x || !codes)) return set_error(kEInval, "bp_encode_bp16: null pointer");
  TRY(check_device());
  return launch_encode_bp16(x, n, rtne != 0, codes, (cudaStream_t)stream);
}

int bp_quire_to_bp32(const uint32_t *limbs, int nlimbs, size_t n, uint32_t *out, void *stream) {
  g_err[0] = 0;
  if (nlimbs != 8 && nlimbs != 12 && nlimbs != 16)
    return set_error(kEInval, "bp_quire_to_bp32: nlimbs must be 8, 12 or 16 (got %d)", nlimbs);
  if (n && (!limbs || !out)) return set_error(kEInval, "bp_quire_to_bp32: null pointer");
  TRY(check_device());
  return launch_quire_to_bp32(limbs, nlimbs, n, out, (cudaStream_t)stream);
}

int bp_quire_to_bp16(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out, void *stream) {
  g_err[0] = 0;
  if (nlimbs != 8 && nlimbs != 12 && nlimbs != 16)
    return set_error(kEInval, "bp_quire_to_bp16: nlimbs must be 8, 12 or 16 (got %d)", nlimbs);
  if (n && (!limbs || !out)) return set_error(kEInval, "bp_quire_to_bp16: null pointer");
  TRY(check_device());
  return launch_quire_to_bp16(limbs, nlimbs, n, out, (cudaStream_t)stream);
}

int bp_bp32_to_bp16(const uint32_t *codes, size_t n, uint16_t *out, void *stream) {
  g_err[0] = 0;
  if (n && (!codes || !out)) return set_error(kEInval, "bp_bp32_to_bp16: null pointer");
  TRY(check_device());
  return launch_bp32_to_bp16(codes, n, out, (cudaStream_t)stream);
}

int bp_quantize_small(int fmt, const double *x, size_t n, uint8_t *codes, void *stream) {
  g_err[0] = 0;
  if (fmt != 4 && fmt != 5) return set_error(kEFmt, "bp_quantize_small: fmt must be 4 or 5 (got %d)", fmt);
  if (n && (!x || !codes)) return set_error(kEInval, "bp_quantize_small: null pointer");
  TRY(check_device());
  return launch_quantize_small(fmt, x, n, codes, (cudaStream_t)stream);
}

int bp_transcode(int fmt_in, int fmt_out, const void *codes, size_t n, void *out, void *stream) {
  g_err[0] = 0;
  if ((fmt_in != 4 && fmt_in != 5 && fmt_in != 8) || (fmt_out != 8 && fmt_out != 16) || fmt_out <= fmt_in)
    return set_error(kEFmt, "bp_transcode: unsupported %d -> %d (4, 5 -> 8, 16; 8 -> 16)", fmt_in, fmt_out);
  if (n && (!codes || !out)) return set_error(kEInval, "bp_transcode: null pointer");
  TRY(check_device());
  return launch_transcode(fmt_in, fmt_out, codes, n, out, (cudaStream_t)stream);
}

size_t bp_quire_gemm_workspace_size(int fmt, int M, int N, int K, int algo) {
  if ((fmt != 8 && fmt != 16) || M < 0 || N < 0 || K < 0) return 0;
  return gemm_workspace_size(fmt, M, N, K, algo);
}

int bp_quire_gemm(int fmt, const void *A, const void *B, int M, int N, int K, const int32_t *sa,
                  const int32_t *sb, int group, uint32_t *out_bp32, int64_t ldo, uint32_t *out_quire,
                  int quire_limbs, int algo, void *workspace, size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_quire_gemm: fmt must be 8 or 16 (got %d)", fmt);
  if (M < 0 || N < 0 || K < 0) return set_error(kEInval, "bp_quire_gemm: negative size");
  if (algo < 0 || algo > 5) return set_error(kEInval, "bp_quire_gemm: algo must be 0 to 5");
  if ((sa || sb) && group <= 0) return set_error(kEInval, "bp_quire_gemm: group must be > 0 with scales");
  if (ldo < N) return set_error(kEInval, "bp_quire_gemm: ldo (%lld) < N (%d)", (long long)ldo, N);
  if (out_quire && quire_limbs != 8 && quire_limbs != 12 && quire_limbs != 16)
    return set_error(kEInval, "bp_quire_gemm: quire_limbs must be 8, 12 or 16");
  if (M == 0 || N == 0) return kOk;
  if (!out_bp32 || (K > 0 && (!A || !B))) return set_error(kEInval, "bp_quire_gemm: null pointer");
  if (workspace && ((uintptr_t)workspace & 255u)) return set_error(kEAlign, "bp_quire_gemm: workspace not 256-byte aligned");
  TRY(check_device());
  GemmArgs a{};
  a.fmt = fmt; a.A = A; a.B = B; a.M = M; a.N = N; a.K = K;
  a.sa = sa; a.sb = sb; a.group = group > 0 ? group : 1;
  a.G = group > 0 ? (K + group - 1) / group : 1;
  a.out = out_bp32; a.ldo = ldo; a.quire = out_quire; a.nlimbs = out_quire ? quire_limbs : 0;
  cudaStream_t s = (cudaStream_t)stream;
  size_t need = gemm_workspace_size(fmt, M, N, K, algo);
  if (workspace) {
    if (workspace_bytes < need)
      return set_error(kEWorkspace, "bp_quire_gemm: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return launch_quire_gemm(a, algo, workspace, workspace_bytes, s);
  }
  void *ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, need, s);
  if (e != cudaSuccess) return set_error(kECuda, "bp_quire_gemm: workspace allocation: %s", cudaGetErrorString(e));
  int rc = launch_quire_gemm(a, algo, ws, need, s);
  cudaError_t f = cudaFreeAsync(ws, s);
  if (rc == kOk && f != cudaSuccess) rc = set_error(kECuda, "bp_quire_gemm: workspace free: %s", cudaGetErrorString(f));
  return rc;
}

int bp_quire_gemm_f32(int fmt, const void *A, const void *B, int M, int N, int K, const int32_t *sa,
                      const int32_t *sb, int group, const int32_t *row_exp, const int32_t *col_exp,
                      const float *bias, float *out_f32, int64_t ldf, uint32_t *out_bp32, int64_t ldo, int algo,
                      void *workspace, size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_quire_gemm_f32: fmt must be 8 or 16 (got %d)", fmt);
  if (M < 0 || N < 0 || K < 0) return set_error(kEInval, "bp_quire_gemm_f32: negative size");
  if (algo < 0 || algo > 5) return set_error(kEInval, "bp_quire_gemm_f32: algo must be 0 to 5");
  if ((sa || sb) && group <= 0) return set_error(kEInval, "bp_quire_gemm_f32: group must be > 0 with scales");
  if (ldf < N) return set_error(kEInval, "bp_quire_gemm_f32: ldf (%lld) < N (%d)", (long long)ldf, N);
  if (out_bp32 && ldo < N) return set_error(kEInval, "bp_quire_gemm_f32: ldo (%lld) < N (%d)", (long long)ldo, N);
  if (M == 0 || N == 0) return kOk;
  if (!out_f32 || (K > 0 && (!A || !B))) return set_error(kEInval, "bp_quire_gemm_f32: null pointer");
  if (workspace && ((uintptr_t)workspace & 255u))
    return set_error(kEAlign, "bp_quire_gemm_f32: workspace not 256-byte aligned");
  TRY(check_device());
  GemmArgs a{};
  a.fmt = fmt; a.A = A; a.B = B; a.M = M; a.N = N; a.K = K;
  a.sa = sa; a.sb = sb; a.group = group > 0 ? group : 1;
  a.G = group > 0 ? (K + group - 1) / group : 1;
  a.out = out_bp32; a.ldo = out_bp32 ? ldo : 0;
  a.out_f32 = out_f32; a.ldf = ldf; a.re = row_exp; a.ce = col_exp; a.bias = bias;
  cudaStream_t s = (cudaStream_t)stream;
  size_t need = gemm_workspace_size(fmt, M, N, K, algo);
  if (workspace) {
    if (workspace_bytes < need)
      return set_error(kEWorkspace, "bp_quire_gemm_f32: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return launch_quire_gemm(a, algo, workspace, workspace_bytes, s);
  }
  void *ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, need, s);
  if (e != cudaSuccess)
    return set_error(kECuda, "bp_quire_gemm_f32: workspace allocation: %s", cudaGetErrorString(e));
  int rc = launch_quire_gemm(a, algo, ws, need, s);
  cudaError_t f = cudaFreeAsync(ws, s);
  if (rc == kOk && f != cudaSuccess) rc = set_error(kECuda, "bp_quire_gemm_f32: workspace free: %s", cudaGetErrorString(f));
  return rc;
}

int bp_quire_gemm_multi(int fmt, const void *A, const void *B, int M, int N, int K, const int32_t *sa,
                        const int32_t *sb, int group, uint32_t *out_bp32, int64_t ldo,
                        uint32_t *const *peer_outs, int n_peer, int64_t peer_col0, int algo, void *workspace,
                        size_t workspace_bytes, void *stream) {
  g_err[0] = 0;
  if (n_peer < 0 || n_peer > kMaxExtraOut)
    return set_error(kEInval, "bp_quire_gemm_multi: n_peer must be in [0, %d]", kMaxExtraOut);
  if (n_peer && (!peer_outs || peer_col0 < 0 || peer_col0 + N > ldo))
    return set_error(kEInval, "bp_quire_gemm_multi: bad peer outputs");
  for (int e = 0; e < n_peer; ++e)
    if (!peer_outs[e]) return set_error(kEInval, "bp_quire_gemm_multi: null peer output %d", e);
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_quire_gemm_multi: fmt must be 8 or 16 (got %d)", fmt);
  if (M < 0 || N < 0 || K < 0) return set_error(kEInval, "bp_quire_gemm_multi: negative size");
  if (algo < 0 || algo > 5) return set_error(kEInval, "bp_quire_gemm_multi: algo must be 0 to 5");
  if ((sa || sb) && group <= 0) return set_error(kEInval, "bp_quire_gemm_multi: group must be > 0 with scales");
  if (ldo < N) return set_error(kEInval, "bp_quire_gemm_multi: ldo (%lld) < N (%d)", (long long)ldo, N);
  if (M == 0 || N == 0) return kOk;
  if (!out_bp32 || (K > 0 && (!A || !B))) return set_error(kEInval, "bp_quire_gemm_multi: null pointer");
  if (workspace && ((uintptr_t)workspace & 255u)) return set_error(kEAlign, "bp_quire_gemm_multi: workspace not 256-byte aligned");
  TRY(check_device());
  GemmArgs a{};
  a.fmt = fmt; a.A = A; a.B = B; a.M = M; a.N = N; a.K = K;
  a.sa = sa; a.sb = sb; a.group = group > 0 ? group : 1;
  a.G = group > 0 ? (K + group - 1) / group : 1;
  a.out = out_bp32; a.ldo = ldo; a.quire = nullptr; a.nlimbs = 0;
  cudaStream_t s = (cudaStream_t)stream;
  const bool tc = gemm_uses_tc(a, algo);
  if (tc) {
    a.n_extra = n_peer; a.extra_col0 = peer_col0;
    for (int e = 0; e < n_peer; ++e) a.extra_out[e] = peer_outs[e];
  }
  size_t need = gemm_workspace_size(fmt, M, N, K, algo);
  void *ws = workspace;
  if (ws && workspace_bytes < need)
    return set_error(kEWorkspace, "bp_quire_gemm_multi: workspace %zu bytes < %zu needed", workspace_bytes, need);
  if (!ws) {
    cudaError_t e = cudaMallocAsync(&ws, need, s);
    if (e != cudaSuccess) return set_error(kECuda, "bp_quire_gemm_multi: workspace allocation: %s", cudaGetErrorString(e));
  }
  int rc = launch_quire_gemm(a, algo, ws, need, s);
  if (rc == kOk && !tc) {   // CUDA-core path: copy the finished block to each peer
    for (int e = 0; e < n_peer && rc == kOk; ++e) {
      cudaError_t ce = cudaMemcpy2DAsync(peer_outs[e] + peer_col0, (size_t)ldo * 4, out_bp32, (size_t)ldo * 4,
                                         (size_t)N * 4, (size_t)M, cudaMemcpyDeviceToDevice, s);
      if (ce != cudaSuccess) rc = set_error(kECuda, "bp_quire_gemm_multi: peer copy: %s", cudaGetErrorString(ce));
    }
  }
  if (!workspace) cudaFreeAsync(ws, s);
  return rc;
}

int bp_quire_gemm_host(int fmt, const void *A, const void *B, int M, int N, int K, const int32_t *sa,
                       const int32_t *sb, int group, uint32_t *out_bp32, int64_t ldo, int algo, void *stream) {
  g_err[0] = 0;
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_quire_gemm_host: fmt must be 8 or 16 (got %d)", fmt);
  if (M < 0 || N < 0 || K < 0) return set_error(kEInval, "bp_quire_gemm_host: negative size");
  if (algo < 0 || algo > 5) return set_error(kEInval, "bp_quire_gemm_host: algo must be 0 to 5");
  if ((sa || sb) && group <= 0) return set_error(kEInval, "bp_quire_gemm_host: group must be > 0 with scales");
  if (ldo < N) return set_error(kEInval, "bp_quire_gemm_host: ldo (%lld) < N (%d)", (long long)ldo, N);
  if (M == 0 || N == 0) return kOk;
  if (!out_bp32 || (K > 0 && (!A || !B))) return set_error(kEInval, "bp_quire_gemm_host: null pointer");
  TRY(check_device());
  return launch_quire_gemm_host(fmt, A, B, M, N, K, sa, sb, group, out_bp32, ldo, algo, (cudaStream_t)stream);
}

int bp_w8a8_encode_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, void *stream) {
  g_err[0] = 0;
  if (rows < 0 || K < 0) return set_error(kEInval, "bp_w8a8_encode_rows: negative size");
  if ((size_t)rows * K != 0 && (!x || !exps || !codes)) return set_error(kEInval, "bp_w8a8_encode_rows: null pointer");
  TRY(check_device());
  return launch_w8a8_rows(x, rows, K, exps, codes, (cudaStream_t)stream);
}

int bp_enable_peer_access(int peer_device) {
  g_err[0] = 0;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return set_error(kENoDev, "bp_enable_peer_access: no device");
  if (peer_device == cur) return kOk;
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, cur, peer_device);
  if (e != cudaSuccess) return set_error(kECuda, "bp_enable_peer_access: %s", cudaGetErrorString(e));
  if (!can) return set_error(kENoDev, "bp_enable_peer_access: device %d cannot access device %d", cur, peer_device);
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return kOk;
  }
  if (e != cudaSuccess) return set_error(kECuda, "bp_enable_peer_access: %s", cudaGetErrorString(e));
  return kOk;
}

int bp_ipc_alloc(size_t bytes, void **ptr, void *handle_out) {
  g_err[0] = 0;
  if (!ptr || !handle_out || bytes == 0) return set_error(kEInval, "bp_ipc_alloc: bad arguments");
  TRY(check_device());
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_error(kECuda, "bp_ipc_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(kECuda, "bp_ipc_alloc: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == BP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return kOk;
}

int bp_ipc_free(void *ptr) {
  g_err[0] = 0;
  if (!ptr) return kOk;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? kOk : set_error(kECuda, "bp_ipc_free: %s", cudaGetErrorString(e));
}

int bp_ipc_open(const void *handle, void **ptr) {
  g_err[0] = 0;
  if (!handle || !ptr) return set_error(kEInval, "bp_ipc_open: null argument");
  TRY(check_device());
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(kECuda, "bp_ipc_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return kOk;
}

int bp_ipc_close(void *ptr) {
  g_err[0] = 0;
  if (!ptr) return kOk;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? kOk : set_error(kECuda, "bp_ipc_close: %s", cudaGetErrorString(e));
}

int bp_bp32_to_f64(const uint32_t *codes, int M, int N, const int32_t *row_exp, const int32_t *col_exp,
                   double *out, void *stream) {
  g_err[0] = 0;
  if (M < 0 || N < 0) return set_error(kEInval, "bp_bp32_to_f64: negative size");
  if ((size_t)M * N != 0 && (!codes || !out)) return set_error(kEInval, "bp_bp32_to_f64: null pointer");
  TRY(check_device());
  return launch_bp32_to_f64(codes, M, N, row_exp, col_exp, out, (cudaStream_t)stream);
}

int bp_bp32_to_f32(const uint32_t *codes, int M, int N, const int32_t *row_exp, const int32_t *col_exp,
                   const float *bias, float *out, void *stream) {
  g_err[0] = 0;
  if (M < 0 || N < 0) return set_error(kEInval, "bp_bp32_to_f32: negative size");
  if ((size_t)M * N != 0 && (!codes || !out)) return set_error(kEInval, "bp_bp32_to_f32: null pointer");
  TRY(check_device());
  return launch_bp32_to_f32(codes, M, N, row_exp, col_exp, bias, out, (cudaStream_t)stream);
}

}  // extern "C"
