/*
 * bposit_b200.h -- C ABI of the B200 (sm_100a) b-posit W8A8 hot path.
 *
 * Plain pointers, sizes and an opaque CUDA stream (cudaStream_t passed as
 * void*; NULL = the legacy default stream).  Every device pointer must point
 * to memory of the current CUDA device.  Every call is asynchronous on
 * `stream` and returns a status: BP_OK (0) or a negative BP_E* code, with a
 * message in bp_last_error() (thread-local).  No C++ exception crosses the ABI.
 *
 * Library-owned state: the tables each kernel builds in its shared memory;
 * per device, one kernel error word (bp_device_error) and the fixed 1 MiB
 * scratch array of bp_quire_gemm_noalloc; per host thread and device, the
 * device and pinned host buffers that bp_quire_gemm_host keeps for later
 * calls (grown to the largest call, held until exit); the CUDA-IPC mappings
 * made by bp_ipc_open until bp_ipc_close.  Apart from the no-alloc scratch
 * (shared by its calls on a device) and the error word, calls on different
 * streams are independent.
 *
 * Formats: fmt = 8 (bp8: 8-bit posit, eS=2, codes uint8) or 16 (bp16: 16-bit
 * posit, eS=3, codes uint16).  bp32 results are uint32 codes (eS=3).  Quires
 * are two's complement integers with 96 fraction bits stored as
 * little-endian 32-bit limbs.
 *
 * Reference interfaces each entry point replaces (paths relative to the
 * open-bposit project root) are cited per function.
 */
#ifndef BPOSIT_B200_H
#define BPOSIT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BP_OK 0
#define BP_EINVAL (-1)     /* null pointer, negative size, bad group / limb count */
#define BP_EFMT (-2)       /* unsupported format */
#define BP_EALIGN (-3)     /* pointer alignment the call requires is not met */
#define BP_ECUDA (-4)      /* CUDA error (launch or runtime) */
#define BP_ERANGE (-5)     /* size beyond what the call supports */
#define BP_ENODEV (-6)     /* no sm_100 device is current */
#define BP_EWORKSPACE (-7) /* workspace missing or too small */

/* Library version: major * 10000 + minor * 100 + patch. */
int bp_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char *bp_last_error(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads).  Diagnostic; no reference counterpart. */
unsigned long long bp_launch_count(void);

/* Reads and clears the current device's kernel error word: nonzero when a
 * bounded wait inside a kernel of the tensor-core path (the GEMM, its staged
 * finish, the narrow form's tail corrections) gave up.  That kernel then
 * drained its own copies in flight (bounded), released its tensor memory and
 * returned; from then until this call clears the word, every bposit32 output
 * of the tensor-core path (bp_quire_gemm, _multi, _host) is NaR (0x80000000),
 * a code no quire round produces.  The GEMM entry points return before their
 * kernels run, so C callers poll this after synchronizing the stream (the
 * Python API does so wherever it copies results to the host).  Synchronizes
 * with the device.  Diagnostic; no reference counterpart. */
int bp_device_error(int *out);

/* Decode n codes to their exact fp32 values; zero and NaR give +0.0.
 * Replaces bposit_ref.code_value (reference/bposit_ref.py:1022-1025) and the
 * (mantissa, exponent) LUT of bposit_fast._lut (reference/bposit_fast.py:27-43).
 * Both bp8 and bp16 values are exactly representable in fp32. */
int bp_decode(int fmt, const void *codes, size_t n, float *out, void *stream);

/* fp32 -> bp8 codes (and, when `values` is non-NULL, their exact fp32 values).
 * nearest = 1: bposit_fast.quantize_bp8(x, nearest=True) -- round to the
 * nearest grid magnitude, ties toward the smaller magnitude; nearest = 0: the
 * truncating mode (largest magnitude <= |x|).  Nonzero |x| < 2^-24 -> +-minpos;
 * |x| >= 2^24 and +-inf -> +-maxpos; NaN -> NaR (0x80, value NaN).
 * Replaces reference/bposit_fast.py:69-99 plus the value->code map of
 * examples/w8a8_rounding_demo.py:30-31,47-49. */
int bp_quantize_bp8(const float *x, size_t n, int nearest, uint8_t *codes, float *values,
                    void *stream);

/* float64 input variant of bp_quantize_bp8 (the reference's own input dtype,
 * reference/bposit_fast.py:90): identical rounding decisions on the exact
 * float64 value; `values` (optional) receives the float64 quantized values,
 * with +-0 keeping the sign of x as np.sign(x) * 0 does. */
int bp_quantize_bp8_f64(const double *x, size_t n, int nearest, uint8_t *codes, double *values,
                        void *stream);

/* Row-wise grouped bp8 quantization of x[rows, K] (row-major): every run of
 * `group` elements along K of a row shares a power-of-two exponent s, and the
 * code is quantize_bp8(x / 2^s).  compute_scales = 1 computes
 * s = ceil(log2(absmax / 2^maxpos_log2)) (0 for an all-zero group) and writes it
 * to exps[rows, ceil(K / group)]; compute_scales = 0 reads exps.  maxpos_log2 is
 * 24 for bp8's maxpos 2^24 (reference/bposit_ref.py:226-227).  No reference
 * counterpart: composes quantize_bp8 with an exact power-of-two scale. */
int bp_quantize_bp8_grouped(const float *x, int rows, int K, int group, int nearest,
                            int compute_scales, int maxpos_log2, int32_t *exps, uint8_t *codes,
                            void *stream);

/* fp32 -> bp16 codes.  rtne = 1: encode_bposit16(Fraction(x), "rtne"),
 * rtne = 0: encode_bposit16(Fraction(x), "truncate")
 * (reference/bposit_ref.py:382-507).  NaN -> NaR (0x8000), +-inf -> +-maxpos. */
int bp_encode_bp16(const float *x, size_t n, int rtne, uint16_t *codes, void *stream);

/* The activation side of the reference's W8A8 recipe, per row of x[rows, K]
 * (fp32): exps[r] = recommended_exponents (round(log2(ref)), ref = the row's
 * RMS, or its 95th percentile of |x| when that exceeds twice the RMS; 0 for an
 * all-zero row), computed in float64 on the device, and codes[r, :] = the
 * truncating bp8 encode of x[r, :] * 2^-exps[r] with encode_bposit8's float
 * entry zero cut (reference/bposit_quantize.py:46-89,
 * reference/bposit_ref.py:258-270).  The float64 sum of squares is reduced in
 * a different order than numpy's, which can change an exponent only when ref
 * is within an ulp of 2^(k + 1/2) or the percentile within an ulp of 2 RMS. */
int bp_w8a8_encode_rows(const float *x, int rows, int K, int32_t *exps, uint8_t *codes, void *stream);

/* Truncating encode of float64 values to the small rungs, one code per byte:
 * fmt 4 = bposit4 (es 1, encode range 2^+-2), fmt 5 = AI-posit5 (es 1,
 * 2^+-4).  Replaces encode_bposit4 / encode_aiposit5 on floats and
 * quantize_vec (reference/bposit_ref.py:852-866, 899-925, 1017-1019),
 * including the float entry's limit_denominator(10**8) zero cut.  NaN -> NaR. */
int bp_quantize_small(int fmt, const double *x, size_t n, uint8_t *codes, void *stream);

/* Exact transcode of codes to a wider format: fmt_in 4 or 5 (one code per
 * byte) or 8, fmt_out 8 (uint8) or 16 (uint16), fmt_out > fmt_in.  Every
 * value of the narrower formats is a value of the wider one; NaR -> NaR.
 * With it the bp8 / bp16 quire GEMM computes the reference's small-rung and
 * mixed-rung quires: dot_at_precision / dot_quire / matmul_quire for bp4 and
 * aip5 and mixed_precision_sum (reference/bposit_ref.py:995-1035,
 * reference/bposit_fast.py:22,102-176). */
int bp_transcode(int fmt_in, int fmt_out, const void *codes, size_t n, void *out, void *stream);

/* Round n quires (nlimbs = 8, 12 or 16 limbs each) once to bposit32.
 * Replaces bposit_ref.quire256_to_bposit32 (reference/bposit_ref.py:703-722). */
int bp_quire_to_bp32(const uint32_t *limbs, int nlimbs, size_t n, uint32_t *out, void *stream);

/* Round n quires once to bposit16 (truncating, saturating at +-maxpos).
 * Replaces bposit_ref.quire256_to_bposit16 (reference/bposit_ref.py:620-635),
 * the out_fmt="bp16" round of dot / dot_at_precision / mixed_precision_sum
 * (reference/bposit_ref.py:989-992, reference/bposit_fast.py:131-133). */
int bp_quire_to_bp16(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out, void *stream);

/* bposit32 codes produced by a quire round (bp_quire_gemm, bp_quire_to_bp32)
 * to the bposit16 round of the same quires.  Both rounds truncate the same
 * regime/exponent/fraction bit string (es = 3 in both), so this is exact:
 * bp16 = top 15 bits of the bp32 field, saturated the way bp16 saturates.
 * The bp16 output of an exact GEMM is bp_quire_gemm followed by this. */
int bp_bp32_to_bp16(const uint32_t *codes, size_t n, uint16_t *out, void *stream);

/* Exact quire GEMM: for m < M, n < N
 *   q[m,n] = sum_k trunc0( v(A[m,k]) * v(B[n,k]) * 2^(sa[m,k/group] + sb[n,k/group]) * 2^96 )
 *   out_bp32[m * ldo + n] = bposit32 of q[m,n] (one truncating round)
 * A[M,K] and B[N,K] are codes of format fmt, row-major with K contiguous; sa,
 * sb (optional, may be NULL) are int32 per-(row, group) exponents
 * [rows, ceil(K/group)].  If out_quire is non-NULL, the raw quires are also
 * written as [M, N, quire_limbs] (quire_limbs 8, 12 or 16; truncated two's
 * complement).  algo: 0 = auto, 1 = CUDA cores, 2 = tensor cores (tcgen05; paired SMs,
 * cta_group::2, when M > 128), 3 = tensor cores with one SM per output tile,
 * 4 / 5 = tensor cores (paired) with the narrow / wide bp8 digit-plane form
 * (2 base-256 planes over a 15-bit window, or 3 base-128 planes over 20 bits;
 * elements below a row's window are corrected on CUDA cores).  Algos 0, 2 and
 * 3 take the narrow form for unscaled bp8 with K >= 16384, else the wide one;
 * bp16 always uses 4 base-128 planes.  Every algo gives the same result.
 * workspace: device memory of at least bp_quire_gemm_workspace_size() bytes,
 * 256-byte aligned; NULL lets the library take it stream-ordered from the
 * device's default memory pool for the duration of the call.
 * Replaces bposit_fast.dot_quire / dot / matmul_quire
 * (reference/bposit_fast.py:102-176) with the final quire256_to_bposit32 of
 * bposit_ref (reference/bposit_ref.py:703-722) and dot_at_precision
 * (reference/bposit_ref.py:1028-1035). */
int bp_quire_gemm(int fmt, const void *A, const void *B, int M, int N, int K,
                  const int32_t *sa, const int32_t *sb, int group,
                  uint32_t *out_bp32, int64_t ldo, uint32_t *out_quire, int quire_limbs,
                  int algo, void *workspace, size_t workspace_bytes, void *stream);

/* bp_quire_gemm with the hand-off to the next fp32 op of a model written by
 * the GEMM's own output stage:
 *   out_f32[m * ldf + n] = fp32( value(bp32[m,n]) * 2^(row_exp[m] + col_exp[n]) + bias[n] )
 * -- the bposit32 round of the exact quire, its exact value scaled by the
 * power-of-two exponents (each optional, NULL = 0) plus the optional fp32 bias,
 * added in float64 and rounded once to the nearest-even fp32; NaR -> NaN.
 * The same numbers as bp_quire_gemm followed by bp_bp32_to_f32, without the
 * second pass over the [M, N] codes.  out_bp32 is optional (NULL: the codes
 * are not stored).  No raw-quire output; single GPU.  Replaces matmul_quire +
 * quire256_to_bposit32 (reference/bposit_fast.py:136-176,
 * reference/bposit_ref.py:703-722) followed by the rescale of quantize_w8a8
 * (reference/bposit_quantize.py:66-68, 88), in fp32 for a torch model. */
int bp_quire_gemm_f32(int fmt, const void *A, const void *B, int M, int N, int K,
                      const int32_t *sa, const int32_t *sb, int group,
                      const int32_t *row_exp, const int32_t *col_exp, const float *bias,
                      float *out_f32, int64_t ldf, uint32_t *out_bp32, int64_t ldo,
                      int algo, void *workspace, size_t workspace_bytes, void *stream);

/* bp_quire_gemm on HOST buffers: A, B, sa, sb and out_bp32 are host pointers
 * (page-locked memory gives full PCIe bandwidth; pageable memory works,
 * slower).  One operand goes to the device whole and is prepared once; the
 * other is streamed in row chunks (A when M >= N, whose chunks' results are
 * whole rows and leave in one contiguous copy each; else B) while earlier
 * chunks are multiplied and their bposit32 blocks copied back, so the copies
 * in, the tensor-core work and the copies out overlap.  Its device buffers
 * are kept per host thread and device for later calls (they grow to the
 * largest call's sizes, about 1.6 GB for 4096 x 4096 x 65536 bp8, and are
 * held until the process exits); a call waits for the previous call of the
 * same thread on that device, whatever its stream.  The
 * call is asynchronous on `stream` like every other entry point: out_bp32 is
 * complete when the stream is.  Same results as bp_quire_gemm.  Replaces
 * matmul_quire + quire256_to_bposit32 on numpy arrays
 * (reference/bposit_fast.py:136-176, reference/bposit_ref.py:703-722). */
int bp_quire_gemm_host(int fmt, const void *A, const void *B, int M, int N, int K, const int32_t *sa,
                       const int32_t *sb, int group, uint32_t *out_bp32, int64_t ldo, int algo, void *stream);

/* bp_quire_gemm whose bposit32 results are also stored, by the GEMM's finish
 * kernel itself, into n_peer further [M, ldo] matrices at column peer_col0 -- on a
 * multi-GPU node, the full result matrices of the other ranks, reached over
 * NVLink (mapped with bp_ipc_open; peer access from bp_enable_peer_access).  One call both
 * computes this rank's N-shard and all-gathers it: after every rank's call has
 * completed (e.g. behind a collective barrier), every rank holds the whole
 * [M, N_total] bposit32 matrix.  out_bp32 points at this rank's block
 * (its full matrix + peer_col0).  n_peer <= 8; no raw-quire output.
 * Replaces the reference's matmul_quire (reference/bposit_fast.py:136-176)
 * for an N-sharded GEMM; the fused all-gather has no reference counterpart. */
int bp_quire_gemm_multi(int fmt, const void *A, const void *B, int M, int N, int K,
                        const int32_t *sa, const int32_t *sb, int group,
                        uint32_t *out_bp32, int64_t ldo, uint32_t *const *peer_outs, int n_peer,
                        int64_t peer_col0, int algo, void *workspace, size_t workspace_bytes,
                        void *stream);

/* Enable direct access from the current device to peer_device's memory
 * (idempotent).  Multi-GPU plumbing; no reference counterpart. */
int bp_enable_peer_access(int peer_device);

/* Device memory shared between the processes of one node (CUDA IPC), for the
 * result buffers that bp_quire_gemm_multi writes across GPUs.
 *   bp_ipc_alloc  -- zeroed allocation on the current device plus its
 *                    BP_IPC_HANDLE_BYTES-byte handle (pass it to the peers);
 *   bp_ipc_open   -- map a peer's handle into the current device's context
 *                    (peer access enabled as needed); *ptr is a device address
 *                    the current device's kernels may load from and store to;
 *   bp_ipc_close  -- unmap what bp_ipc_open returned;
 *   bp_ipc_free   -- free what bp_ipc_alloc returned (after every peer closed).
 * Multi-GPU plumbing; no reference counterpart. */
#define BP_IPC_HANDLE_BYTES 64
int bp_ipc_alloc(size_t bytes, void **ptr, void *handle_out);
int bp_ipc_free(void *ptr);
int bp_ipc_open(const void *handle, void **ptr);
int bp_ipc_close(void *ptr);

/* Workspace bytes bp_quire_gemm needs for this shape and algo. */
size_t bp_quire_gemm_workspace_size(int fmt, int M, int N, int K, int algo);

/* bp_quire_gemm without any device allocation, for callers that cannot
 * allocate: plugins whose host framework owns the whole device-memory budget,
 * and latency-critical loops where cudaMalloc / cudaFree (which can
 * synchronize the device) are not acceptable.  Same arguments and results as
 * bp_quire_gemm on the CUDA-core path, minus algo and workspace.  Its scratch is
 * a fixed 1 MiB device array inside the library (held by every GPU that loads
 * it, until exit), so M + N must not exceed 65,536 rows (BP_ERANGE otherwise).
 * The first call on each device looks up that array's device address; make it
 * before any stream capture.  All calls on a device share the array: calls
 * that overlap on the GPU race and must be serialized by the caller.
 * No counterpart in the reference (it has no device memory at all). */
int bp_quire_gemm_noalloc(int fmt, const void *A, const void *B, int M, int N, int K,
                          const int32_t *sa, const int32_t *sb, int group,
                          uint32_t *out_bp32, int64_t ldo, uint32_t *out_quire, int quire_limbs,
                          void *stream);

/* bposit32 codes -> float64 values times 2^(row_exp[m] + col_exp[n]) for an
 * [M, N] matrix (row/col exponents may be NULL = 0); NaR -> 0.0 as in
 * _bp32_to_float.  Exact (unless the scaled value leaves the float64 range): bp32
 * values carry at most 28 significant bits.  Replaces the rescale step
 * _bp32_to_float(c) * 2^(ex+ew) of bposit_quantize.quantize_w8a8
 * (reference/bposit_quantize.py:66-68, 88). */
int bp_bp32_to_f64(const uint32_t *codes, int M, int N, const int32_t *row_exp,
                   const int32_t *col_exp, double *out, void *stream);

/* The same values plus an optional fp32 column bias [N], each rounded once to
 * the nearest-even fp32: the hand-off from an exact W8A8 GEMM to the next
 * fp32 op of a model (the nn.Linear drop-in).  NaR -> NaN (no quire round
 * produces NaR; a GEMM that gave up on a bounded wait writes it).  No reference
 * counterpart (the reference stops at float64). */
int bp_bp32_to_f32(const uint32_t *codes, int M, int N, const int32_t *row_exp, const int32_t *col_exp,
                   const float *bias, float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BPOSIT_B200_H */
