// bp_noalloc.cu -- bp_quire_gemm_noalloc: the exact quire GEMM for callers
// that must not allocate device memory.
//
// Who cannot allocate: a plugin running inside a host framework that owns the
// whole device-memory budget (every byte comes from the host's own pools), and
// latency-critical loops where a cudaMalloc / cudaFree -- which can
// synchronize the device -- is not acceptable.  They still pass their own
// inputs and outputs; this entry point needs nothing else.
//
// Its only scratch (the per-row operand statistics of the CUDA-core GEMM) lives
// in a fixed file-scope device array of kNoAllocScratchBytes, which every GPU
// that loads this library holds until the process exits.  In host code the
// array's name is only a host-side stand-in, so the device address is looked up
// with cudaGetSymbolAddress (with that device current) and cached per CUDA
// context: the first call in each context (normally once per device, in its
// primary context) does that set-up and should therefore come before any
// stream capture; a context created later on the same device -- after a
// cudaDeviceReset, say, which unloads the library's module and may move the
// array -- is seen as new and looked up again.  All calls on a device share the
// one array and it keeps the last call's contents: every byte a call reads is
// written by the same call first, but calls that overlap on the GPU (different
// streams, or threads racing on one device) race on it and must be serialized.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/bposit_b200.h"
#include "bp_internal.cuh"

namespace bp {
int launch_gemm_simt(const GemmArgs &a, int4 *sta, int4 *stb, cudaStream_t s);
}  // namespace bp

using namespace bp;

// 1 MiB: one 16-byte statistics record per row of A and of B, so M + N <= 65536.
static constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void *g_noalloc_addr[128];   // per device: the array's address in context g_noalloc_ctx
static CUcontext g_noalloc_ctx[128];

// The driver's cuCtxGetCurrent, resolved once through the runtime (the library
// links only the runtime).
static PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuCtxGetCurrent_v4000)p;
  });
  return fn;
}

// Device address of g_noalloc_scratch on the current device, looked up once per
// context.  When no context is current yet, cudaGetSymbolAddress itself binds
// the device's primary context, which is read back afterwards.
static int noalloc_scratch(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(kENoDev, "bp_quire_gemm_noalloc: no CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(kENoDev, "bp_quire_gemm_noalloc: device index %d out of range", dev);
  auto get_ctx = ctx_get_current();
  if (!get_ctx) return set_error(kECuda, "bp_quire_gemm_noalloc: cuCtxGetCurrent unavailable");
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!ctx || !g_noalloc_addr[dev] || g_noalloc_ctx[dev] != ctx) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(kECuda, "bp_quire_gemm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    if (!ctx && (get_ctx(&ctx) != CUDA_SUCCESS || !ctx))
      return set_error(kECuda, "bp_quire_gemm_noalloc: no CUDA context on device %d", dev);
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_addr[dev];
  return kOk;
}

extern "C" int bp_quire_gemm_noalloc(int fmt, const void *A, const void *B, int M, int N, int K,
                                     const int32_t *sa, const int32_t *sb, int group, uint32_t *out_bp32,
                                     int64_t ldo, uint32_t *out_quire, int quire_limbs, void *stream) {
  clear_error();
  if (fmt != 8 && fmt != 16) return set_error(kEFmt, "bp_quire_gemm_noalloc: fmt must be 8 or 16 (got %d)", fmt);
  if (M < 0 || N < 0 || K < 0) return set_error(kEInval, "bp_quire_gemm_noalloc: negative size");
  if ((sa || sb) && group <= 0) return set_error(kEInval, "bp_quire_gemm_noalloc: group must be > 0 with scales");
  if (ldo < N) return set_error(kEInval, "bp_quire_gemm_noalloc: ldo (%lld) < N (%d)", (long long)ldo, N);
  if (out_quire && quire_limbs != 8 && quire_limbs != 12 && quire_limbs != 16)
    return set_error(kEInval, "bp_quire_gemm_noalloc: quire_limbs must be 8, 12 or 16");
  size_t need = ((size_t)M + (size_t)N) * sizeof(int4);
  if (need > kNoAllocScratchBytes)
    return set_error(kERange,
                     "bp_quire_gemm_noalloc: M + N = %lld rows exceeds the fixed scratch limit of %zu rows "
                     "(use bp_quire_gemm with a workspace)",
                     (long long)M + N, kNoAllocScratchBytes / sizeof(int4));
  if (M == 0 || N == 0) return kOk;
  if (!out_bp32 || (K > 0 && (!A || !B))) return set_error(kEInval, "bp_quire_gemm_noalloc: null pointer");
  int rc = check_device();
  if (rc != kOk) return rc;
  void *scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != kOk) return rc;
  GemmArgs a{};
  a.fmt = fmt; a.A = A; a.B = B; a.M = M; a.N = N; a.K = K;
  a.sa = sa; a.sb = sb; a.group = group > 0 ? group : 1;
  a.G = group > 0 ? (K + group - 1) / group : 1;
  a.out = out_bp32; a.ldo = ldo; a.quire = out_quire; a.nlimbs = out_quire ? quire_limbs : 0;
  cudaStream_t s = (cudaStream_t)stream;
  int4 *sta = (int4 *)scratch;
  int4 *stb = sta + M;
  rc = launch_row_stats2(fmt, A, M, sa, sta, B, N, sb, stb, K, a.group, s);
  if (rc != kOk) return rc;
  return launch_gemm_simt(a, sta, stb, s);
}
