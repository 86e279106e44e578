// bp_host.cu -- the quire GEMM on host buffers, with the copies overlapped.
//
// A (M x K codes) goes to the device whole; B is streamed in row chunks of nc
// rows (nc a multiple of the 96-column tile).  While chunk c is prepared and
// multiplied on the caller's stream, chunk c+1 is copied in on a copy stream
// and chunk c-1's bposit32 block is copied out on another (PCIe is full
// duplex).  A is prepared once, as soon as it is on the device (while B's
// first chunk is still in flight); every chunk reuses its digit planes, bases
// and tail lists (launch_quire_gemm a_mode 2, then 1).  Every chunk
// has the same shape (the last one padded with zero rows, whose outputs are not
// copied out), so every chunk uses the same workspace layout.  The result is
// exactly bp_quire_gemm's: chunks are column blocks and outputs are
// column-independent.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "bp_internal.cuh"

namespace bp {

namespace {

// The library's own stream-ordered pool for this path's buffers (one per
// device).  It keeps freed memory for the next call instead of returning it
// to the driver at every synchronization, which would make every call re-map
// ~1.5 GB of device memory for the 4096 x 4096 x 65536 case.
cudaMemPool_t host_path_pool(int dev) {
  static std::mutex mu;
  static cudaMemPool_t pools[128] = {};
  if (dev < 0 || dev >= 128) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    if (cudaMemPoolCreate(&p, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = p;
  }
  return pools[dev];
}

struct HostPipe {
  cudaStream_t cin = nullptr, cout = nullptr;
  cudaEvent_t ev[16] = {};
  void *buf[8] = {};
  cudaStream_t s = nullptr;
  ~HostPipe() {
    // every buffer is freed in stream order on s after all copy work
    if (s) {
      if (cin && ev[14]) {
        cudaEventRecord(ev[14], cin);
        cudaStreamWaitEvent(s, ev[14], 0);
      }
      if (cout && ev[15]) {
        cudaEventRecord(ev[15], cout);
        cudaStreamWaitEvent(s, ev[15], 0);
      }
      for (void *p : buf)
        if (p) cudaFreeAsync(p, s);
    }
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    if (cin) cudaStreamDestroy(cin);
    if (cout) cudaStreamDestroy(cout);
  }
};

}  // namespace

int launch_quire_gemm_host(int fmt, const void *A_h, const void *B_h, int M, int N, int K, const int32_t *sa_h,
                           const int32_t *sb_h, int group, uint32_t *out_h, int64_t ldo, int algo,
                           cudaStream_t s) {
  const size_t es = (size_t)fmt / 8;
  const int G = (sa_h || sb_h) ? (K + group - 1) / group : 1;
  // chunk B when there is enough data for the overlap to pay
  const size_t bytes = ((size_t)M + N) * K * es;
  int nch = bytes >= (size_t)64 << 20 ? std::max(1, std::min(4, N / 384)) : 1;
  const int nc = (((N + nch - 1) / nch) + 95) / 96 * 96;
  nch = (N + nc - 1) / nc;
  const int ncw = nch > 1 ? nc : N;   // rows of every chunk buffer (and the GEMM's N)

  HostPipe hp;
  hp.s = s;
  cudaError_t e = cudaSuccess;
  auto ck = [&](cudaError_t r, const char *what) {
    if (r != cudaSuccess && e == cudaSuccess) {
      e = r;
      set_error(kECuda, "quire_gemm_host: %s: %s", what, cudaGetErrorString(r));
    }
    return r == cudaSuccess;
  };
  if (!ck(cudaStreamCreateWithFlags(&hp.cin, cudaStreamNonBlocking), "stream")) return kECuda;
  if (!ck(cudaStreamCreateWithFlags(&hp.cout, cudaStreamNonBlocking), "stream")) return kECuda;
  for (cudaEvent_t &ev : hp.ev)
    if (!ck(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event")) return kECuda;
  cudaEvent_t evStart = hp.ev[0], evA = hp.ev[1];
  cudaEvent_t *evB = hp.ev + 2, *evG = hp.ev + 4, *evO = hp.ev + 6;

  GemmArgs a{};
  a.fmt = fmt; a.M = M; a.N = ncw; a.K = K; a.group = group > 0 ? group : 1; a.G = G;
  const size_t need_ws = gemm_workspace_size(fmt, M, ncw, K, algo);
  void *&dA = hp.buf[0], *&ws = hp.buf[1], *&dsa = hp.buf[2];
  void **dB = hp.buf + 3, **dO = hp.buf + 5;   // two of each
  void *&dsb_all = hp.buf[7];
  auto sz = [](size_t v) { return std::max<size_t>(v, 256); };
  int dev = 0;
  cudaGetDevice(&dev);
  cudaMemPool_t pool = host_path_pool(dev);
  auto alloc = [&](void **p, size_t bytes) {
    return ck(pool ? cudaMallocFromPoolAsync(p, sz(bytes), pool, s) : cudaMallocAsync(p, sz(bytes), s),
              "allocation");
  };
  if (!alloc(&dA, (size_t)M * K * es) || !alloc(&ws, need_ws) || !alloc(&dB[0], (size_t)ncw * K * es) ||
      !alloc(&dB[1], (size_t)ncw * K * es) || !alloc(&dO[0], (size_t)M * ncw * 4) ||
      !alloc(&dO[1], (size_t)M * ncw * 4))
    return kECuda;
  if (sa_h && !alloc(&dsa, (size_t)M * G * 4)) return kECuda;
  if (sb_h && !alloc(&dsb_all, 2 * (size_t)ncw * G * 4)) return kECuda;
  int32_t *dsb[2] = {sb_h ? (int32_t *)dsb_all : nullptr, sb_h ? (int32_t *)dsb_all + (size_t)ncw * G : nullptr};

  // the copies start after everything already queued on the caller's stream
  ck(cudaEventRecord(evStart, s), "event");
  ck(cudaStreamWaitEvent(hp.cin, evStart, 0), "wait");
  ck(cudaStreamWaitEvent(hp.cout, evStart, 0), "wait");
  ck(cudaMemcpyAsync(dA, A_h, (size_t)M * K * es, cudaMemcpyHostToDevice, hp.cin), "copy in");
  if (sa_h) ck(cudaMemcpyAsync(dsa, sa_h, (size_t)M * G * 4, cudaMemcpyHostToDevice, hp.cin), "copy in");
  ck(cudaEventRecord(evA, hp.cin), "event");
  ck(cudaStreamWaitEvent(s, evA, 0), "wait");
  if (e != cudaSuccess) return kECuda;
  a.A = dA; a.B = dB[0]; a.sa = (const int32_t *)dsa; a.sb = dsb[0];
  a.out = (uint32_t *)dO[0]; a.ldo = ncw;
  // prepare A while B's first chunk is still on its way
  int rc = launch_quire_gemm(a, algo, ws, sz(need_ws), s, /*a_mode=*/2);
  if (rc) return rc;

  for (int c = 0; c < nch && rc == kOk; ++c) {
    const int b = c & 1;
    const int n0 = c * nc;
    const int ncc = std::min(nc, N - n0);
    if (c >= 2) ck(cudaStreamWaitEvent(hp.cin, evG[b], 0), "wait");   // chunk c-2 no longer reads dB[b]
    if (ncc < ncw) {
      ck(cudaMemsetAsync((char *)dB[b] + (size_t)ncc * K * es, 0, (size_t)(ncw - ncc) * K * es, hp.cin), "memset");
      if (sb_h) ck(cudaMemsetAsync(dsb[b] + (size_t)ncc * G, 0, (size_t)(ncw - ncc) * G * 4, hp.cin), "memset");
    }
    ck(cudaMemcpyAsync(dB[b], (const char *)B_h + (size_t)n0 * K * es, (size_t)ncc * K * es,
                       cudaMemcpyHostToDevice, hp.cin), "copy in");
    if (sb_h)
      ck(cudaMemcpyAsync(dsb[b], sb_h + (size_t)n0 * G, (size_t)ncc * G * 4, cudaMemcpyHostToDevice, hp.cin),
         "copy in");
    ck(cudaEventRecord(evB[b], hp.cin), "event");
    ck(cudaStreamWaitEvent(s, evB[b], 0), "wait");
    if (c >= 2) ck(cudaStreamWaitEvent(s, evO[b], 0), "wait");      // chunk c-2's block has left dO[b]
    if (e != cudaSuccess) return kECuda;
    a.A = dA; a.B = dB[b]; a.sa = (const int32_t *)dsa; a.sb = dsb[b];
    a.out = (uint32_t *)dO[b]; a.ldo = ncw;
    rc = launch_quire_gemm(a, algo, ws, sz(need_ws), s, /*a_mode=*/1);
    if (rc) break;
    ck(cudaEventRecord(evG[b], s), "event");
    ck(cudaStreamWaitEvent(hp.cout, evG[b], 0), "wait");
    ck(cudaMemcpy2DAsync(out_h + n0, (size_t)ldo * 4, dO[b], (size_t)ncw * 4, (size_t)ncc * 4, (size_t)M,
                         cudaMemcpyDeviceToHost, hp.cout), "copy out");
    ck(cudaEventRecord(evO[b], hp.cout), "event");
    if (e != cudaSuccess) return kECuda;
  }
  // the caller's stream completes after the last block is on the host
  // (HostPipe's destructor joins both copy streams into s, then frees)
  return rc;
}

}  // namespace bp
