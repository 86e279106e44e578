// bp_host.cu -- the quire GEMM on host buffers, with the copies overlapped.
//
// One operand goes to the device whole and is prepared once; the other is
// streamed in row chunks (a multiple of the tile), each chunk copied in on a
// copy stream while the previous one is multiplied on the caller's stream, and
// each chunk's bposit32 block copied out on another copy stream (PCIe is full
// duplex).  Every chunk has the same shape (the last one padded with zero rows,
// whose outputs are not copied out), so every chunk uses the same workspace
// layout and reuses the whole operand's digit planes, bases and tail lists
// (launch_quire_gemm a_mode 2 then 1, or 3 then 4).  The result is exactly
// bp_quire_gemm's: outputs are independent of one another.
//
//  * M >= N: B whole, A streamed in row chunks.  A chunk's outputs are whole
//    rows of the result, so they leave in one contiguous copy.
//  * M < N: A whole, B streamed in row chunks; a chunk's outputs are a column
//    block of the result, copied out row by row (a 2-D copy).  Measured on
//    B200, a 2-D copy of 4 KB rows moves 10 GB/s against 57 GB/s contiguous,
//    which is why the row-chunked form is preferred when it has the rows.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "bp_internal.cuh"

namespace bp {

namespace {

// Device buffers of this path, kept per thread and device for later calls
// (they grow to the largest call's sizes and are never returned): allocating
// ~1.5 GB per call for the 4096 x 4096 x 65536 case -- even from a
// stream-ordered pool, whose allocation calls took 14-33 ms of host time per
// call on B200 -- cost more than the copies.  `done` is recorded on the
// caller's stream at the end of each call; the next call waits for it, so
// calls on different streams never overlap on these buffers.
struct HostBuffers {
  void *p[8] = {};
  size_t cap[8] = {};
  cudaEvent_t done = nullptr;
};

HostBuffers *host_buffers() {
  constexpr int kDev = 64;
  thread_local HostBuffers hb[kDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDev) {
    cudaGetLastError();
    return nullptr;
  }
  return &hb[dev];
}

struct HostPipe {
  cudaStream_t cin = nullptr, cout = nullptr;
  cudaEvent_t ev[16] = {};
  void *buf[8] = {};
  HostBuffers *hb = nullptr;
  cudaStream_t s = nullptr;
  bool started = false;   // work was queued: the copy streams are joined into s
  ~HostPipe() {
    if (s && started) {
      if (cin && ev[14]) {
        cudaEventRecord(ev[14], cin);
        cudaStreamWaitEvent(s, ev[14], 0);
      }
      if (cout && ev[15]) {
        cudaEventRecord(ev[15], cout);
        cudaStreamWaitEvent(s, ev[15], 0);
      }
      if (hb && hb->done) cudaEventRecord(hb->done, s);
    }
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    if (cin) cudaStreamDestroy(cin);
    if (cout) cudaStreamDestroy(cout);
  }
  // Buffer `slot` with at least `bytes` bytes (256 at least), grown if needed.
  cudaError_t alloc(int slot, size_t bytes) {
    bytes = std::max<size_t>(bytes, 256);
    if (hb->cap[slot] < bytes) {
      if (hb->p[slot]) {
        if (hb->done) cudaEventSynchronize(hb->done);   // no earlier call still uses it
        cudaFree(hb->p[slot]);
        hb->p[slot] = nullptr;
        hb->cap[slot] = 0;
      }
      cudaError_t e = cudaMalloc(&hb->p[slot], bytes);
      if (e != cudaSuccess) {
        hb->p[slot] = nullptr;
        return e;
      }
      hb->cap[slot] = bytes;
    }
    buf[slot] = hb->p[slot];
    return cudaSuccess;
  }
  // Set-up shared by both forms: buffers, copy streams, events, and the wait
  // for the previous call on these buffers.
  cudaError_t open(cudaStream_t stream) {
    s = stream;
    hb = host_buffers();
    if (!hb) return cudaErrorInvalidDevice;
    cudaError_t e = cudaSuccess;
    if (!hb->done) e = cudaEventCreateWithFlags(&hb->done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cin, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cout, cudaStreamNonBlocking);
    for (cudaEvent_t &x : ev)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&x, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, hb->done, 0);
    return e;
  }
};

}  // namespace

namespace {

// A whole, B streamed in row chunks (column blocks of the result).
int host_cols(int fmt, const void *A_h, const void *B_h, int M, int N, int K, const int32_t *sa_h,
              const int32_t *sb_h, int group, uint32_t *out_h, int64_t ldo, int algo, cudaStream_t s) {
  const size_t es = (size_t)fmt / 8;
  const int G = (sa_h || sb_h) ? (K + group - 1) / group : 1;
  // chunk B when there is enough data for the overlap to pay
  const size_t bytes = ((size_t)M + N) * K * es;
  int nch = bytes >= (size_t)64 << 20 ? std::max(1, std::min(4, N / 384)) : 1;
  const int nc = (((N + nch - 1) / nch) + 95) / 96 * 96;
  nch = (N + nc - 1) / nc;
  const int ncw = nch > 1 ? nc : N;   // rows of every chunk buffer (and the GEMM's N)

  HostPipe hp;
  cudaError_t e = cudaSuccess;
  auto ck = [&](cudaError_t r, const char *what) {
    if (r != cudaSuccess && e == cudaSuccess) {
      e = r;
      set_error(kECuda, "quire_gemm_host: %s: %s", what, cudaGetErrorString(r));
    }
    return r == cudaSuccess;
  };
  if (!ck(hp.open(s), "set-up")) return kECuda;
  cudaEvent_t evStart = hp.ev[0], evA = hp.ev[1];
  cudaEvent_t *evB = hp.ev + 2, *evG = hp.ev + 4, *evO = hp.ev + 6;

  GemmArgs a{};
  a.fmt = fmt; a.M = M; a.N = ncw; a.K = K; a.group = group > 0 ? group : 1; a.G = G;
  const size_t need_ws = std::max<size_t>(gemm_workspace_size(fmt, M, ncw, K, algo), 256);
  // slots: 0 A, 1 workspace, 2 sa, 3-4 B chunks, 5-6 result blocks, 7 sb chunks
  if (!ck(hp.alloc(0, (size_t)M * K * es), "allocation") || !ck(hp.alloc(1, need_ws), "allocation") ||
      !ck(hp.alloc(3, (size_t)ncw * K * es), "allocation") || !ck(hp.alloc(4, (size_t)ncw * K * es), "allocation") ||
      !ck(hp.alloc(5, (size_t)M * ncw * 4), "allocation") || !ck(hp.alloc(6, (size_t)M * ncw * 4), "allocation"))
    return kECuda;
  if (sa_h && !ck(hp.alloc(2, (size_t)M * G * 4), "allocation")) return kECuda;
  if (sb_h && !ck(hp.alloc(7, 2 * (size_t)ncw * G * 4), "allocation")) return kECuda;
  void *dA = hp.buf[0], *ws = hp.buf[1], *dsa = sa_h ? hp.buf[2] : nullptr;
  void **dB = hp.buf + 3, **dO = hp.buf + 5;
  void *dsb_all = hp.buf[7];
  hp.started = true;
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
  int rc = launch_quire_gemm(a, algo, ws, need_ws, s, /*a_mode=*/2);
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
    rc = launch_quire_gemm(a, algo, ws, need_ws, s, /*a_mode=*/1);
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

// B whole, A streamed in row chunks (row blocks of the result).
int host_rows(int fmt, const void *A_h, const void *B_h, int M, int N, int K, const int32_t *sa_h,
              const int32_t *sb_h, int group, uint32_t *out_h, int64_t ldo, int algo, cudaStream_t s) {
  const size_t es = (size_t)fmt / 8;
  const int G = (sa_h || sb_h) ? (K + group - 1) / group : 1;
  // chunk A when there is enough data for the overlap to pay; chunks of whole
  // 256-row tile pairs
  const size_t bytes = ((size_t)M + N) * K * es;
  int nch = bytes >= (size_t)64 << 20 ? std::max(1, std::min(4, M / 512)) : 1;
  const int mc = (((M + nch - 1) / nch) + 255) / 256 * 256;
  nch = (M + mc - 1) / mc;
  const int mcw = nch > 1 ? mc : M;   // rows of every chunk buffer (and the GEMM's M)

  HostPipe hp;
  cudaError_t e = cudaSuccess;
  auto ck = [&](cudaError_t r, const char *what) {
    if (r != cudaSuccess && e == cudaSuccess) {
      e = r;
      set_error(kECuda, "quire_gemm_host: %s: %s", what, cudaGetErrorString(r));
    }
    return r == cudaSuccess;
  };
  if (!ck(hp.open(s), "set-up")) return kECuda;
  cudaEvent_t evStart = hp.ev[0], evB = hp.ev[1];
  cudaEvent_t *evA = hp.ev + 2, *evG = hp.ev + 4, *evO = hp.ev + 6;

  GemmArgs a{};
  a.fmt = fmt; a.M = mcw; a.N = N; a.K = K; a.group = group > 0 ? group : 1; a.G = G;
  const size_t need_ws = std::max<size_t>(gemm_workspace_size(fmt, mcw, N, K, algo), 256);
  // slots: 0 B, 1 workspace, 2 sb, 3-4 A chunks, 5-6 result blocks, 7 sa chunks
  if (!ck(hp.alloc(0, (size_t)N * K * es), "allocation") || !ck(hp.alloc(1, need_ws), "allocation") ||
      !ck(hp.alloc(3, (size_t)mcw * K * es), "allocation") || !ck(hp.alloc(4, (size_t)mcw * K * es), "allocation") ||
      !ck(hp.alloc(5, (size_t)mcw * N * 4), "allocation") || !ck(hp.alloc(6, (size_t)mcw * N * 4), "allocation"))
    return kECuda;
  if (sb_h && !ck(hp.alloc(2, (size_t)N * G * 4), "allocation")) return kECuda;
  if (sa_h && !ck(hp.alloc(7, 2 * (size_t)mcw * G * 4), "allocation")) return kECuda;
  void *dB = hp.buf[0], *ws = hp.buf[1], *dsb = sb_h ? hp.buf[2] : nullptr;
  void **dA = hp.buf + 3, **dO = hp.buf + 5;
  void *dsa_all = hp.buf[7];
  hp.started = true;
  int32_t *dsa[2] = {sa_h ? (int32_t *)dsa_all : nullptr, sa_h ? (int32_t *)dsa_all + (size_t)mcw * G : nullptr};

  // the copies start after everything already queued on the caller's stream
  ck(cudaEventRecord(evStart, s), "event");
  ck(cudaStreamWaitEvent(hp.cin, evStart, 0), "wait");
  ck(cudaStreamWaitEvent(hp.cout, evStart, 0), "wait");
  ck(cudaMemcpyAsync(dB, B_h, (size_t)N * K * es, cudaMemcpyHostToDevice, hp.cin), "copy in");
  if (sb_h) ck(cudaMemcpyAsync(dsb, sb_h, (size_t)N * G * 4, cudaMemcpyHostToDevice, hp.cin), "copy in");
  ck(cudaEventRecord(evB, hp.cin), "event");
  ck(cudaStreamWaitEvent(s, evB, 0), "wait");
  if (e != cudaSuccess) return kECuda;
  a.A = dA[0]; a.B = dB; a.sa = dsa[0]; a.sb = (const int32_t *)dsb;
  a.out = (uint32_t *)dO[0]; a.ldo = N;
  // prepare B while A's first chunk is still on its way
  int rc = launch_quire_gemm(a, algo, ws, need_ws, s, /*a_mode=*/3);
  if (rc) return rc;

  for (int c = 0; c < nch && rc == kOk; ++c) {
    const int b = c & 1;
    const int m0 = c * mc;
    const int mcc = std::min(mc, M - m0);
    if (c >= 2) ck(cudaStreamWaitEvent(hp.cin, evG[b], 0), "wait");   // chunk c-2 no longer reads dA[b]
    if (mcc < mcw) {
      ck(cudaMemsetAsync((char *)dA[b] + (size_t)mcc * K * es, 0, (size_t)(mcw - mcc) * K * es, hp.cin), "memset");
      if (sa_h) ck(cudaMemsetAsync(dsa[b] + (size_t)mcc * G, 0, (size_t)(mcw - mcc) * G * 4, hp.cin), "memset");
    }
    ck(cudaMemcpyAsync(dA[b], (const char *)A_h + (size_t)m0 * K * es, (size_t)mcc * K * es,
                       cudaMemcpyHostToDevice, hp.cin), "copy in");
    if (sa_h)
      ck(cudaMemcpyAsync(dsa[b], sa_h + (size_t)m0 * G, (size_t)mcc * G * 4, cudaMemcpyHostToDevice, hp.cin),
         "copy in");
    ck(cudaEventRecord(evA[b], hp.cin), "event");
    ck(cudaStreamWaitEvent(s, evA[b], 0), "wait");
    if (c >= 2) ck(cudaStreamWaitEvent(s, evO[b], 0), "wait");      // chunk c-2's block has left dO[b]
    if (e != cudaSuccess) return kECuda;
    a.A = dA[b]; a.B = dB; a.sa = dsa[b]; a.sb = (const int32_t *)dsb;
    a.out = (uint32_t *)dO[b]; a.ldo = N;
    rc = launch_quire_gemm(a, algo, ws, need_ws, s, /*a_mode=*/4);
    if (rc) break;
    ck(cudaEventRecord(evG[b], s), "event");
    ck(cudaStreamWaitEvent(hp.cout, evG[b], 0), "wait");
    if (ldo == N)
      ck(cudaMemcpyAsync(out_h + (size_t)m0 * N, dO[b], (size_t)mcc * N * 4, cudaMemcpyDeviceToHost, hp.cout),
         "copy out");
    else
      ck(cudaMemcpy2DAsync(out_h + (size_t)m0 * ldo, (size_t)ldo * 4, dO[b], (size_t)N * 4, (size_t)N * 4,
                           (size_t)mcc, cudaMemcpyDeviceToHost, hp.cout), "copy out");
    ck(cudaEventRecord(evO[b], hp.cout), "event");
    if (e != cudaSuccess) return kECuda;
  }
  // the caller's stream completes after the last block is on the host
  // (HostPipe's destructor joins both copy streams into s, then frees)
  return rc;
}

}  // namespace

int launch_quire_gemm_host(int fmt, const void *A_h, const void *B_h, int M, int N, int K, const int32_t *sa_h,
                           const int32_t *sb_h, int group, uint32_t *out_h, int64_t ldo, int algo,
                           cudaStream_t s) {
  return M >= N ? host_rows(fmt, A_h, B_h, M, N, K, sa_h, sb_h, group, out_h, ldo, algo, s)
                : host_cols(fmt, A_h, B_h, M, N, K, sa_h, sb_h, group, out_h, ldo, algo, s);
}

}  // namespace bp
