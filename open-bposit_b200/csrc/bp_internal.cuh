// bp_internal.cuh -- launch helpers shared by the library's .cu files.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "bp_format.cuh"

namespace bp {

// Status codes (mirrored in include/bposit_b200.h).
enum {
  kOk = 0,
  kEInval = -1,
  kEFmt = -2,
  kEAlign = -3,
  kECuda = -4,
  kERange = -5,
  kENoDev = -6,
  kEWorkspace = -7,
};

int set_error(int code, const char *fmt, ...);
void clear_error();    // empties this host thread's bp_last_error() message
int check_device();    // kENoDev unless the current device is an sm_100 GPU
int check_launch(const char *what);
int sm_count();   // SMs of the current device

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0u; }

// ---- codec launchers (bp_codec.cu) ----
int launch_decode(int fmt, const void *codes, size_t n, float *out, cudaStream_t s);
int launch_quantize_bp8(const float *x, size_t n, bool nearest, uint8_t *codes, float *values,
                        cudaStream_t s);
int launch_quantize_bp8_f64(const double *x, size_t n, bool nearest, uint8_t *codes, double *values,
                            cudaStream_t s);
int launch_encode_bp16(const float *x, size_t n, bool rtne, uint16_t *codes, cudaStream_t s);
int launch_group_quantize_bp8(const float *x, int rows, int K, int group, bool nearest,
                              bool compute_scales, int maxpos_log2, int32_t *exps, uint8_t *codes,
                              cudaStream_t s);
int launch_quantize_small(int fmt, const double *x, size_t n, uint8_t *codes, cudaStream_t s);
int launch_transcode(int fmt_in, int fmt_out, const void *codes, size_t n, void *out, cudaStream_t s);
int launch_bp32_to_f32(const uint32_t *codes, int M, int N, const int32_t *re, const int32_t *ce,
                       const float *bias, float *out, cudaStream_t s);
int launch_quire_gemm_host(int fmt, const void *A_h, const void *B_h, int M, int N, int K, const int32_t *sa_h,
                           const int32_t *sb_h, int group, uint32_t *out_h, int64_t ldo, int algo,
                           cudaStream_t s);
int launch_w8a8_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, cudaStream_t s);
int launch_quire_to_bp16(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out, cudaStream_t s);
int launch_bp32_to_bp16(const uint32_t *codes, size_t n, uint16_t *out, cudaStream_t s);
int launch_quire_to_bp32(const uint32_t *limbs, int nlimbs, size_t n, uint32_t *out,
                         cudaStream_t s);

// ---- quire GEMM (bp_gemm_simt.cu, bp_gemm_tc.cu) ----
constexpr int kMaxExtraOut = 8;
struct GemmArgs {
  int fmt;                 // 8 or 16
  const void *A, *B;       // [M,K], [N,K] codes, K contiguous
  int M, N, K;
  const int32_t *sa, *sb;  // per-(row, group) exponents or null
  int group, G;
  uint32_t *out;           // bp32 codes, row stride ldo (may be null when out_f32 is set)
  int64_t ldo;
  // Optional fp32 hand-off written by the GEMM's own output stage:
  // out_f32[i * ldf + j] = fp32(value(bp32) * 2^(re[i] + ce[j]) + bias[j])
  // (re, ce, bias optional); single-GPU calls only (no extra outputs).
  float *out_f32;
  int64_t ldf;
  const int32_t *re, *ce;
  const float *bias;
  // Extra destinations (tensor-core path): every bp32 word is also stored at
  // extra_out[r][i * ldo + extra_col0 + j] -- e.g. the full result matrices of
  // peer GPUs, written over NVLink by the GEMM epilogue.
  uint32_t *extra_out[kMaxExtraOut];
  int n_extra;
  int64_t extra_col0;
  uint32_t *quire;         // optional raw quires [M, N, nlimbs]
  int nlimbs;
};

size_t gemm_workspace_size(int fmt, int M, int N, int K, int algo);
bool gemm_uses_tc(const GemmArgs &a, int algo);
// a_mode (tensor-core path): 0 prepare A and B, then multiply; 1 reuse A's
// preparation from an earlier call on the same workspace; 2 prepare A only;
// 3 prepare B only; 4 reuse B's preparation.
int launch_quire_gemm(const GemmArgs &a, int algo, void *ws, size_t ws_bytes, cudaStream_t s,
                      int a_mode = 0);
// Row statistics {min lsb exponent, max binade, nonzero} of both operands in one launch.
int launch_row_stats2(int fmt, const void *codes, int rows, const int32_t *s, int4 *stats, const void *codes2,
                      int rows2, const int32_t *s2, int4 *stats2, int K, int group, cudaStream_t st);

}  // namespace bp
