// bp_rungs.cu -- the small precision rungs of the unified quire: bposit4
// (es 1) and AI-posit5 (es 1) (reference/bposit_ref.py:879-940).
//
// Every bposit4 / AI-posit5 value is exactly a bposit8 value, and every
// bposit8 value exactly a bposit16 value, so a mixed-rung quire sum or dot
// (mixed_precision_sum, dot_at_precision, reference/bposit_ref.py:995-1035)
// is the bp8 (or bp16) quire GEMM on transcoded codes: the transcode is exact
// and the quire terms are the same numbers.  Transcoding is a 16/32/256-entry
// table lookup built per block in shared memory from the format decoders.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_format.cuh"
#include "bp_internal.cuh"

namespace bp {
namespace {

constexpr int kThreads = 256;

inline int grid_for(size_t n) {
  size_t b = (n + kThreads - 1) / kThreads;
  size_t cap = (size_t)sm_count() * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

template <int NB, int ES, int MAXE>
__global__ void __launch_bounds__(kThreads) k_quantize_small(const double *__restrict__ x, size_t n,
                                                             uint8_t *__restrict__ codes) {
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) codes[i] = (uint8_t)small_encode<NB, ES, MAXE>(x[i]);
}

// The transcode table entry for input code c: the output-format code of the
// same value (NaR -> NaR, zero -> zero).
template <int NBI, int ESI, bool OUT16>
__device__ uint32_t transcode_entry(uint32_t c) {
  Dec d = decode_posit<NBI, ESI>(c);
  if (d.kind == 1) return 0u;
  if (d.kind == 2) return OUT16 ? 0x8000u : 0x80u;
  const uint32_t v = posit_to_f32_bits<NBI, ESI>(c);
  if constexpr (OUT16) {
    return bp16_encode_bits(v, true);   // exact value: either mode gives its code
  } else {
    for (uint32_t c8 = 1; c8 < 256; ++c8)
      if (c8 != 0x80u && posit_to_f32_bits<8, 2>(c8) == v) return c8;
    return 0x80u;   // unreachable: every small-rung value is a bp8 value
  }
}

template <int NBI, int ESI, bool OUT16>
__global__ void __launch_bounds__(kThreads) k_transcode(const uint8_t *__restrict__ in, size_t n,
                                                        void *__restrict__ out) {
  __shared__ uint16_t lut[1 << NBI];
  for (uint32_t c = threadIdx.x; c < (1u << NBI); c += blockDim.x)
    lut[c] = (uint16_t)transcode_entry<NBI, ESI, OUT16>(c);
  __syncthreads();
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n; i += stride) {
    const uint16_t v = lut[in[i] & ((1u << NBI) - 1u)];
    if (OUT16) ((uint16_t *)out)[i] = v;
    else ((uint8_t *)out)[i] = (uint8_t)v;
  }
}

template <int NBI, int ESI>
void transcode_launch(const uint8_t *in, size_t n, void *out, bool out16, cudaStream_t s) {
  if (out16) k_transcode<NBI, ESI, true><<<grid_for(n), kThreads, 0, s>>>(in, n, out);
  else k_transcode<NBI, ESI, false><<<grid_for(n), kThreads, 0, s>>>(in, n, out);
}

}  // namespace

int launch_quantize_small(int fmt, const double *x, size_t n, uint8_t *codes, cudaStream_t s) {
  if (n == 0) return kOk;
  if (fmt == 4) k_quantize_small<4, 1, 2><<<grid_for(n), kThreads, 0, s>>>(x, n, codes);
  else k_quantize_small<5, 1, 4><<<grid_for(n), kThreads, 0, s>>>(x, n, codes);
  return check_launch("quantize_small");
}

int launch_transcode(int fmt_in, int fmt_out, const void *codes, size_t n, void *out, cudaStream_t s) {
  if (n == 0) return kOk;
  const uint8_t *in = (const uint8_t *)codes;
  const bool out16 = fmt_out == 16;
  if (fmt_in == 4) transcode_launch<4, 1>(in, n, out, out16, s);
  else if (fmt_in == 5) transcode_launch<5, 1>(in, n, out, out16, s);
  else transcode_launch<8, 2>(in, n, out, out16, s);
  return check_launch("transcode");
}

}  // namespace bp
