// bp_gemm_tc.cu -- exact quire GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in TMEM, operands staged by TMA).
//
// Same result as the CUDA-core path (and as dot_at_precision /
// bposit_fast.matmul_quire + quire256_to_bposit32, reference/bposit_ref.py:1028-1035,
// reference/bposit_fast.py:102-176, reference/bposit_ref.py:703-722), computed by
// exponent-sliced integer MMAs:
//
//  1. k_tc_prep, one block per operand row r: row statistics (min lsb exponent
//     la_r, max binade hb_r), then a main base L_r = max(la_r, hb_r - SPAN + 1).
//     Every element with lsb >= L_r is an integer X = v / 2^L_r, |X| < 2^SPAN,
//     recoded into S signed base-128 digits X = sum_s d_s 128^s (low digits in
//     [-64, 63], top digit |d| <= 65) and stored as S int8 planes
//     [S][rows][Kp].  bp8: S = 3, SPAN = 20; bp16: S = 4, SPAN = 27.  The rare
//     elements below L_r (a row's far tail) are listed instead.
//  2. k_tc_corr adds the tails back exactly on CUDA cores:
//     A_tail * B + A_main * B_tail, one 128-bit sum per touched output.
//  3. k_quire_gemm_tc issues, per 64-deep K block, S*S*2 int8 MMAs
//     (128 x BN x 32) and accumulates digit pair (s, t) into TMEM accumulator
//     d = s + t; the S MMAs sharing an A digit plane reuse it from the tensor
//     core's A collector.  With base-128 digits a diagonal grows by at most
//     12416 (bp8) / 16512 (bp16) per k, so int32 stays exact for K up to
//     KCHUNK; longer K is cut into chunks summed by k_tc_finish.
//  4. The epilogue reads the 2S-1 diagonals and stores Q = sum_d acc_d * 128^d
//     exactly (one int64 word for bp8, two for bp16); k_tc_finish adds the K
//     chunks, moves Q to the output's lsb base la_i + la_j, adds the tail
//     correction and rounds once to bposit32.
//  5. Outputs whose exact window exceeds 128 bits, that need per-term
//     truncation (products below 2^-96), or whose tail list overflowed are
//     recomputed by k_tc_fixup with the 512-bit quire of the CUDA-core slow
//     path (it exits at once when global row bounds show there are none).
//
// Warp roles in the GEMM (128 threads, one CTA per SM, 512 TMEM columns):
// warp 0 lane 0 issues TMA loads, warps 1 and 2 issue the MMAs of alternate
// K blocks, all four warps run the epilogue (warp w reads TMEM lanes
// 32w..32w+31 = tile rows).  All mbarrier waits are bounded; a timeout sets an
// error word and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <mutex>
#include <type_traits>

#include "bp_gemm_common.cuh"
#include "bp_internal.cuh"

namespace bp {

__device__ int g_tc_error;   // nonzero after a bounded wait gave up

namespace {

#ifndef BP_TC_BK
#define BP_TC_BK 64
#endif
constexpr int BM = 128, BK = BP_TC_BK, THREADS = 256;
constexpr long long WAIT_LIMIT = 4000000000LL;   // cycles (~2 s) before a wait gives up
constexpr long long DRAIN_LIMIT = 200000000LL;   // cycles (~0.1 s) per stage drained after a timeout
constexpr int TAILCAP = 1024;                    // listed tail elements per row (more -> fixup)
constexpr int BIG = 1 << 20;                     // offset that makes max-reductions find a minimum

// Tile configuration.  PAIR: the 2-SM form -- a cluster of two CTAs issues
// M = 256 MMAs (tcgen05 cta_group::2); each CTA holds its own 128 rows of A and
// half of the tile's B rows, and owns 128 rows of the output tile.
// S = 2 is the narrow bp8 form: two base-256 digits (low digit in [-128, 127])
// over a 15-bit main window; a bp8 significand has at most 4 bits, so |X| <=
// 2^15 - 2^11 and the top digit stays within [-120, 120].  S = 3 (bp8) and
// S = 4 (bp16) are the wide forms, base-128 digits (low digits in [-64, 63]).
template <int S, bool PAIR = false>
struct Cfg {
  static constexpr int DB = S == 2 ? 8 : 7;        // bits per digit
  static constexpr int BN = S == 2 ? 128 : (S == 3 ? 96 : 64);
  static constexpr int BNB = PAIR ? BN / 2 : BN;   // B rows (tile columns) staged by one CTA
  static constexpr int MM = PAIR ? 2 * BM : BM;    // rows of one MMA
  static constexpr int D = 2 * S - 1;
  static constexpr int SPAN = S == 2 ? 15 : 7 * S - 1;
  static constexpr int HALF = 1 << (DB - 1);       // low digits lie in [-HALF, HALF)
  static constexpr int TOP = S == 2 ? ((1 << 15) - (1 << 11) + HALF) >> 8
                                    : (1 << (SPAN - 7 * (S - 1))) + 1;   // bound of |top digit|
  static constexpr long long digit_max(int s) { return s == S - 1 ? TOP : HALF; }
  static constexpr long long diag_bound(int d) {
    long long b = 0;
    for (int s = 0; s < S; ++s)
      if (d - s >= 0 && d - s < S) b += digit_max(s) * digit_max(d - s);
    return b;
  }
  static constexpr long long max_diag() {
    long long m = 0;
    for (int d = 0; d < D; ++d) m = diag_bound(d) > m ? diag_bound(d) : m;
    return m;
  }
  // K per chunk with every int32 diagonal sum exact, a multiple of BK
  static constexpr int KCHUNK = (int)((0x7FFFFFFFLL / max_diag()) / BK * BK);
  // int64 words per exact main sum handed to k_tc_finish: bp8 (D = 5) one,
  // Q = sum_d acc_d 128^d with |Q| < 2^31 * 2^28 * 1.01 < 2^60; bp16 (D = 7)
  // two, lo = sum_{d<4} acc_d 128^d (< 2^53) and hi = sum_{d>=4} acc_d
  // 128^(d-4) (< 2^46), Q = lo + hi * 2^28, which may need up to 74 bits.
  // S = 2: Q = acc_0 + acc_1 2^8 + acc_2 2^16, |Q| < 2^48, one word.
  static constexpr int QW = D <= 5 ? 1 : 2;
  static constexpr int A_BYTES = S * BM * BK;
  static constexpr int B_BYTES = S * BNB * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // (S = 2 paired: 7 stages, 177 KB, leave room on the SM for the narrow form's
  // copy and correction blocks that run beside the GEMM)
  static constexpr int STAGES = PAIR ? (S == 2 ? 7 : (S == 3 ? 6 : 5))
                                     : (BK == 128 ? 2 : (S == 2 ? 6 : (S == 3 ? 5 : 4)));
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + BN * 32;
  static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(MM >> 4) << 24);
  static_assert(D * BN <= 512, "TMEM budget");
  static_assert(BN % 32 == 0 && BN <= 256, "UMMA N");
  static_assert(BNB % 8 == 0, "B rows per CTA in whole 8-row swizzle atoms");
  static_assert(!PAIR || BK == 64, "the paired form uses 64-deep K blocks");
  static_assert(STAGE_BYTES % 1024 == 0, "stages stay 1 KB aligned");
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(TOP <= 127, "top digit must fit int8");
  static_assert(KCHUNK >= BK, "at least one K block per exact chunk");
};

// Per-operand device counters, zeroed before each call:
//   v[0] correction slots used, v[1] tail-list entries used, v[8] (side A)
//   the narrow form's correction work counter,
//   v[2] BIG - min la over nonzero rows, v[3] max (hb - la), v[4] any row whose
//   tail could not be listed, v[5] any nonzero row.
struct TcCounters {
  int v[16];
};

struct TcParams {
  int M, N, K, Kp, nkb, kb_per_chunk;
  int tile0, ntn;              // first linear tile of this launch; tiles along N
  int ntl;                     // tiles of this launch
  int split;                   // K chunks per tile in this launch (1: whole tiles)
  const int4 *sta, *stb;
  const int *LA, *LB, *slotA, *slotB;
  const ulonglong2 *CA, *CB;   // tail corrections [slot][other dim], 128-bit
  uint32_t *out;               // may be null when out_f32 is set
  int64_t ldo;
  float *out_f32;              // optional fp32 hand-off (GemmArgs::out_f32), row stride ldf
  int64_t ldf;
  const int32_t *re, *ce;
  const float *bias;
  uint32_t *quire;
  int nlimbs;
  long long *qbuf;             // [tile - tile0][chunk][MM rows][BN cols]: exact main sums Q (int64)
  uint32_t *extra_out[kMaxExtraOut];   // peer result matrices (row stride ldo)
  int n_extra;
  int64_t extra_col0;
};

// ---------------------------------------------------------------- PTX ---
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  A timeout records `code` in g_tc_error and raises the CTA's
// abort word, which makes every other bounded wait of the CTA give up at once.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int code,
                                          volatile int *abort = nullptr, bool nap = false) {
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (nap) __nanosleep(256);   // idle warps keep off the shared-memory pipe
    if (abort && *abort) return false;
    if (clock64() - t0 > WAIT_LIMIT) {
      atomicOr(&g_tc_error, code);
      if (abort) *abort = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// The TMA load of the paired form: the destination is this CTA's shared
// memory, the completion goes to `bar`, a shared::cluster address (the pair
// leader's barrier).  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs of the cluster; release/acquire orders shared
// memory (barrier initialisation, epilogue reads) across the pair.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of `p`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_smem(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

template <bool PAIR>
__device__ __forceinline__ void tmem_alloc_t(uint32_t *slot, uint32_t ncols) {
  if (PAIR) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  } else {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
}

template <bool PAIR>
__device__ __forceinline__ void tmem_dealloc_t(uint32_t taddr, uint32_t ncols) {
  if (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
  else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile with 64-byte swizzle: rows of 64 bytes (BK int8),
// 8-row atoms 512 bytes apart (SBO), leading offset 16 bytes (unused by the
// swizzle), descriptor version 1, layout SWIZZLE_64B.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  if (BK == 128)
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)32 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// D[tmem] (+)= A[adesc] . B[bdesc]^T, int8 x int8 -> int32, issued by one
// lane elected from the calling (converged) warp so that the whole issue loop
// stays warp-uniform.  COL selects the A-collector use: 0 load A and keep it,
// 1 reuse the kept A, 2 reuse and release, 3 no collector.
#define BP_UMMA_ASM(GROUP, QUAL)                                                            \
  asm volatile(                                                                             \
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"    \
      "@e tcgen05.mma.cta_group::" GROUP ".kind::i8" QUAL " [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d), \
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate))

template <int COL, bool PAIR = false>
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  if (PAIR) {
    if (COL == 0) BP_UMMA_ASM("2", ".collector::a::fill");
    else if (COL == 1) BP_UMMA_ASM("2", ".collector::a::use");
    else if (COL == 2) BP_UMMA_ASM("2", ".collector::a::lastuse");
    else BP_UMMA_ASM("2", "");
  } else {
    if (COL == 0) BP_UMMA_ASM("1", ".collector::a::fill");
    else if (COL == 1) BP_UMMA_ASM("1", ".collector::a::use");
    else if (COL == 2) BP_UMMA_ASM("1", ".collector::a::lastuse");
    else BP_UMMA_ASM("1", "");
  }
}
#undef BP_UMMA_ASM

// Arrive on `bar` once every tcgen05 operation this warp issued so far has
// completed (one elected lane commits).
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// The paired form's commit: arrive on `bar` in both CTAs of the pair (the
// same shared-memory offset in each; cta mask 0b11) once every tcgen05
// operation this warp issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}\n"
      ::"r"(smem_u32(bar)), "h"((unsigned short)3)
      : "memory");
}

// Warp-uniform bounded wait: every lane leaves together once any lane has
// seen the phase complete (completion is monotonic).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, int code,
                                               volatile int *abort = nullptr) {
  long long t0 = clock64();
  while (true) {
    bool done = mbar_try_wait(bar, parity);
    if (__any_sync(0xFFFFFFFFu, done)) return true;
    if (abort && __any_sync(0xFFFFFFFFu, *abort != 0)) return false;
    if (clock64() - t0 > WAIT_LIMIT) {
      if ((threadIdx.x & 31) == 0) {
        atomicOr(&g_tc_error, code);
        if (abort) *abort = 1;
      }
      return false;
    }
  }
}

// Abort path of the TMA producer: wait, bounded and without the abort
// shortcut, for the completion of the last round issued on each stage, so
// that no bulk copy still writes this CTA's shared memory once it exits.
// `remote` (the paired form's second CTA, whose copies complete on the
// leader's barriers): sleep a settle time instead.
template <int STAGES>
__device__ __noinline__ void drain_loads(uint64_t *full, uint32_t first, uint32_t end, bool remote) {
  if (remote) {
    for (int i = 0; i < 400; ++i) __nanosleep(1000);   // ~0.4 ms
    return;
  }
  // loads [first, end) of the ring's running count; the last round of each stage
  for (uint32_t g = end - first > (uint32_t)STAGES ? end - STAGES : first; g < end; ++g) {
    const long long t0 = clock64();
    const uint32_t par = (g / STAGES) & 1u;
    while (!mbar_try_wait(&full[g % STAGES], par) && clock64() - t0 < DRAIN_LIMIT) __nanosleep(256);
  }
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ unsigned __int128 u128(ulonglong2 v) {
  return ((unsigned __int128)v.y << 64) | v.x;
}

// Is the TC result of output (i, j) exact (else k_tc_fixup recomputes it)?
__device__ __forceinline__ bool tc_exact(int4 ra, int4 rb, int slot_i, int slot_j, int K) {
  return ra.x + rb.x + 96 >= 0 && fast_width(ra, rb, K, 0) <= 127 && slot_i != -2 && slot_j != -2;
}

// Final bposit32 of output (i, j) from its main-part sum Q (lsb base L_i +
// L_j); the raw quire limbs, when requested, are stored here too.  Returns
// false when the output is left to k_tc_fixup.
__device__ __forceinline__ bool finish_code(const TcParams &p, int i, int j, unsigned __int128 Q, int4 ra,
                                            int4 rb, int Li, int Lj, int slot_i, int slot_j, uint32_t &code) {
  uint32_t *oq = p.quire ? p.quire + ((size_t)i * p.N + j) * p.nlimbs : nullptr;
  if (!(ra.z && rb.z)) {
    if (oq)
      for (int t = 0; t < p.nlimbs; ++t) oq[t] = 0u;
    code = 0u;
    return true;
  }
  if (!tc_exact(ra, rb, slot_i, slot_j, p.K)) return false;
  int sh = (Li - ra.x) + (Lj - rb.x);
  unsigned __int128 tot = Q << sh;
  if (slot_i >= 0) tot += u128(p.CA[(size_t)slot_i * p.N + j]);
  if (slot_j >= 0) tot += u128(p.CB[(size_t)slot_j * p.M + i]);
  code = write_fast_output(tot, ra.x + rb.x + 96, nullptr, oq, p.nlimbs);
  return true;
}

// Tile order: groups of kTileGroup tile rows, M fastest inside a group, so
// that the tiles of one wave (consecutive indices) cover a compact block of
// the output -- 8 tile rows x ~10 tile columns for a 74-pair wave -- and the
// digit-plane slices they read at the same K position are shared in L2 by
// more CTAs (an N-fastest order made every wave read all of B's planes).
// A bijection of [0, ntm * ntn) onto the tile grid.
constexpr int kTileGroup = 8;

__device__ __forceinline__ void tile_coords(int tile, int ntm, int ntn, int &tm, int &tn) {
  const int per_group = kTileGroup * ntn;
  const int g = tile / per_group;
  const int first = g * kTileGroup;
  const int gs = min(ntm - first, kTileGroup);
  const int r = tile - g * per_group;
  tm = first + r % gs;
  tn = r / gs;
}

// ----------------------------------------------------------------- GEMM ---
// One CTA per SM.  PAIR: launched in clusters of two; CTA rank 0 (the leader)
// issues M = 256 MMAs that read A from both CTAs (128 rows each) and B from
// both (half of the tile's columns each) and write each CTA's own TMEM.
template <int S, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    k_quire_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    TcParams p) {
  using C = Cfg<S, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t *empty = full + C::STAGES;
  uint64_t *tfull = empty + C::STAGES;
  uint32_t *tmem_slot = (uint32_t *)(tfull + 1);
  volatile int *abort = (volatile int *)(tmem_slot + 1);                  // set by a timed-out wait

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;      // 0: issues the pair's MMAs

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 2);   // one commit from each issuing warp (of the leader, when paired)
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (PAIR) cluster_sync_all();   // the peer's barriers exist before anything reaches them
  if (warp == 0) tmem_alloc_t<PAIR>(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Persistent: the CTA (pair) takes work units u = (tile, K chunk) of this
  // launch, u = cta, cta + ncta, ...; the stage ring's phases run on across
  // units (gk: K blocks of this CTA's earlier units), tfull completes once per
  // unit.  A unit's epilogue stages its sums in the pipeline buffers, so the
  // next unit's loads start after the whole CTA (pair) has finished it.
  const int cta = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ncta = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int nunits = p.ntl * p.split;
  uint32_t gk = 0, ucount = 0;
  for (int u = cta; u < nunits; u += ncta, ++ucount) {
    const int tl = u / p.split, chunk = u - tl * p.split;
    const int tile = p.tile0 + tl;
    int tm, tn;
    tile_coords(tile, (p.M + C::MM - 1) / C::MM, p.ntn, tm, tn);
    const int n0 = tn * C::BN;
    const int m0 = tm * C::MM + (int)rank * BM;
    const int kb0 = chunk * p.kb_per_chunk;
    const int kb1 = min(p.nkb, kb0 + p.kb_per_chunk);
    const int nkb = kb1 - kb0;
    bool ok = true;

    if (warp == 0) {
      if (lane == 0) {
        int issued = 0;   // K blocks of this unit whose loads were issued
        for (int it = 0; it < nkb && ok; ++it) {
          const uint32_t g = gk + (uint32_t)it;
          const int st = (int)(g % C::STAGES);
          const uint32_t round = g / C::STAGES;
          ok = mbar_wait(&empty[st], (round & 1u) ^ 1u, 1, abort);
          if (!ok) break;
          issued = it + 1;
          uint8_t *sa = smem + st * C::STAGE_BYTES;
          if (PAIR) {
            // both CTAs' loads complete on the leader's barrier, which expects both
            if (rank == 0) mbar_expect_tx(&full[st], 2 * C::STAGE_BYTES);
            const uint32_t fb = cluster_smem(&full[st], 0);
            tma_load_3d_pair(sa, &tmA, fb, (kb0 + it) * BK, m0, 0);
            tma_load_3d_pair(sa + C::A_BYTES, &tmB, fb, (kb0 + it) * BK, n0 + (int)rank * C::BNB, 0);
          } else {
            mbar_expect_tx(&full[st], C::STAGE_BYTES);
            tma_load_3d(sa, &tmA, &full[st], (kb0 + it) * BK, m0, 0);
            tma_load_3d(sa + C::A_BYTES, &tmB, &full[st], (kb0 + it) * BK, n0, 0);
          }
        }
        // After a timeout, the loads still in flight land before this CTA
        // releases its shared memory: wait (bounded, regardless of the abort
        // word) for the last issued round of every stage.  In the paired form
        // the leader's barriers count both CTAs' bytes; the other CTA, whose
        // loads complete on the leader's barriers, waits a settle time instead.
        if (!ok || *abort) drain_loads<C::STAGES>(full, gk, gk + (uint32_t)issued, PAIR && rank != 0);
      }
      __syncwarp();
    } else if ((warp == 1 || warp == 2) && rank == 0) {
      // Two issuing warps take alternate K blocks of the unit.  A warp waits for
      // its block's data while the other warp issues, then takes the hand-off
      // (named barrier 1 or 2 between the two warps, bracketed by tcgen05
      // fences so the MMAs of consecutive blocks stay ordered in the tensor
      // pipe): the full-barrier poll, which stalls MMA issue for ~200 cycles
      // when the issuing warp does it, is off the critical path.  Every
      // iteration takes the same hand-off steps whether or not its wait
      // succeeded, so a timeout cannot strand the partner at a named barrier;
      // each unit's hand-offs pair up within the unit.
      const int me = warp - 1;
      uint32_t init = me ? (1u << C::D) - 1u : 0u;   // block 0 (warp 1) initialises every diagonal
      for (int it = me; it < nkb; it += 2) {
        const uint32_t g = gk + (uint32_t)it;
        const int st = (int)(g % C::STAGES);
        const uint32_t round = g / C::STAGES;
        if (ok) ok = mbar_wait_warp(&full[st], round & 1u, 2, abort);
        if (it > 0) {
          asm volatile("bar.sync %0, 64;" ::"r"(1 + me) : "memory");
          tc_fence_after();
        }
        if (ok) {
          uint32_t a0 = smem_u32(smem + st * C::STAGE_BYTES);
          uint32_t b0 = a0 + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 32; ++ks) {
#pragma unroll
            for (int s = 0; s < S; ++s) {
              uint64_t ad = sw64_desc(a0 + s * BM * BK + ks * 32);
#pragma unroll
              for (int t = 0; t < S; ++t) {
                const int d = s + t;
                uint64_t bd = sw64_desc(b0 + t * C::BNB * BK + ks * 32);
                const uint32_t acc = (init >> d) & 1u;
                if (t == 0) umma_i8<0, PAIR>(tmem + d * C::BN, ad, bd, C::IDESC, acc);
                else if (t == S - 1) umma_i8<2, PAIR>(tmem + d * C::BN, ad, bd, C::IDESC, acc);
                else umma_i8<1, PAIR>(tmem + d * C::BN, ad, bd, C::IDESC, acc);
                init |= 1u << d;
              }
            }
          }
          if (PAIR) {   // the slot is free in both CTAs
            umma_commit_pair(&empty[st]);
          } else {
            umma_commit(&empty[st]);
          }
        }
        if (it + 1 < nkb) {
          tc_fence_before();
          asm volatile("bar.arrive %0, 64;" ::"r"(1 + (me ^ 1)) : "memory");
        }
      }
      if (PAIR) {
        umma_commit_pair(tfull);
      } else {
        umma_commit(tfull);
      }
      __syncwarp();
    }

    // ---------------------------------------------------------------- epilogue
    // Eight warps: warp w reads TMEM lane quarter w & 3 (tile rows 32q..32q+31,
    // the only lanes its tcgen05.ld may touch) and column half w >> 2.
    // The issuing warps commit to tfull whether or not they aborted, so this wait
    // (bounded, but not cut short by the abort word) also drains every MMA in
    // flight before TMEM is read or released.
    ok = mbar_wait(tfull, ucount & 1u, 4, nullptr, true) && ok && !*abort;
    tc_fence_after();
    const int q4 = warp & 3, half = warp >> 2;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    // The epilogue only moves the exact main sums out (Q = sum_d acc_d 2^(DB d),
    // in Cfg::QW int64 words) -- staged per lane quarter in the idle pipeline
    // buffers, [32 rows][BN + 1] int64 per word, conflict-free both ways -- and
    // stores them row by row (coalesced) into this launch's tile-compact buffer.
    // Rounding, tail corrections and the stores of the bposit32 outputs run in
    // k_tc_finish at full occupancy: done here, with one CTA of 8 warps per SM,
    // they took a third to three quarters of a short-K tile's time.
    constexpr int CW = C::BN / 2, QW = C::QW, STG = 4 * 32 * (C::BN + 1);
    static_assert(C::BN % 32 == 0 && CW % 16 == 0, "BN must be a multiple of 32");
    static_assert(QW * STG * 8 <= C::STAGES * C::STAGE_BYTES, "staging fits the pipeline");
    long long *stg = (long long *)smem + q4 * 32 * (C::BN + 1);
#pragma unroll 1
    for (int c0 = half * CW; c0 < half * CW + CW; c0 += 16) {
      uint32_t v[C::D][16];
#pragma unroll
      for (int d = 0; d < C::D; ++d) tmem_ld16(trow + d * C::BN + c0, v[d]);
      tmem_ld_wait();
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        long long lo = 0, hi = 0;
#pragma unroll
        for (int d = 0; d < C::D; ++d) {
          if (QW == 1 || d < 4) lo += (long long)(int)v[d][jj] * (1ll << (C::DB * d));
          else hi += (long long)(int)v[d][jj] * (1ll << (C::DB * (d - 4)));
        }
        stg[lane * (C::BN + 1) + c0 + jj] = lo;
        if (QW == 2) stg[STG + lane * (C::BN + 1) + c0 + jj] = hi;
      }
    }
    {
      // the two warps of a lane quarter meet, then each stores half of its rows
      asm volatile("bar.sync %0, 64;" ::"r"(3 + q4) : "memory");
      long long *dst = p.qbuf + ((size_t)tl * p.split + chunk) * QW * C::MM * C::BN +
                       (size_t)(rank * BM + q4 * 32) * C::BN;
      if (ok) {
#pragma unroll 1
        for (int rr = half * 16; rr < half * 16 + 16; ++rr) {
#pragma unroll
          for (int w = 0; w < QW; ++w)
#pragma unroll
            for (int qq = 0; qq < C::BN / 32; ++qq) {
              const int cc = qq * 32 + lane;
              dst[(size_t)w * C::MM * C::BN + (size_t)rr * C::BN + cc] = stg[w * STG + rr * (C::BN + 1) + cc];
            }
        }
      }
    }
    gk += (uint32_t)nkb;
    // the staging above (generic proxy) before the next unit's loads (async
    // proxy) into the same buffers; TMEM reads before the next unit's MMAs
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    if (PAIR) cluster_sync_all();
    else __syncthreads();
    tc_fence_after();
    // A CTA that gave up on a bounded wait takes no further units, nor does its
    // partner: both read both abort words after the barrier (every wait of the
    // unit has ended by then, so the words are final and both CTAs agree).
    bool stop = *abort != 0;
    if (PAIR) {
      uint32_t peer;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(peer) : "r"(cluster_smem((const void *)abort, rank ^ 1u)));
      stop = stop || peer != 0u;
    }
    if (stop) break;
  }
  if (p.n_extra) __threadfence_system();   // peer stores complete before the kernel does
  tc_fence_before();
  if (PAIR) cluster_sync_all();   // both CTAs are done with the pair's TMEM
  else __syncthreads();
  if (warp == 0) tmem_dealloc_t<PAIR>(tmem, 512);
  if (PAIR) cluster_sync_all();   // neither CTA leaves while the other still deallocates
}

// --------------------------------------------------------------- finish ---
// The outputs of a launch's tiles: the exact main sum Q (the K chunks' sums,
// QW int64 words each), moved to the output's lsb base, plus the tail
// corrections, rounded once to bposit32 and stored (to the output and every
// extra output).
//
// A block takes items -- 1/parts of a tile's rows, all its columns -- in a
// grid-stride loop; lane l owns the columns l, l + 32, ..., whose statistics
// it loads once per item; warp w takes the item's rows w, w + 8, ...  While
// the chunk sums stay inside int64 (always, but for a raw quire output or
// more than 8 bp8 K chunks) a lane adds its sums in int64 and rounds the plain
// ones (no tail correction, nonzero row and column, inside the exact window)
// with the short builder; the others of the row load all their tail
// corrections at once and take finish_code's 128-bit rule.  With one K chunk
// the loads of the warp's next row are issued before the current row is
// rounded (software pipelining: the loads' latency was the kernel's main
// stall).  Otherwise every output goes through finish_general one by one.

// The general rule for output (i, j) of a unit: the chunks' sums added in 128
// bits, finish_code (tail corrections, zero rows, raw quire), stores.
template <int QW, bool F32>
__device__ __forceinline__ void finish_general(const TcParams &p, const long long *a, size_t plane, int i, int j) {
  __int128 Q = 0;
  for (int ch = 0; ch < p.split; ++ch) {
    const long long *ac = a + (size_t)ch * QW * plane;
    Q += (__int128)__ldcs(ac);
    if (QW == 2) Q += (__int128)__ldcs(ac + plane) << 28;
  }
  uint32_t code;
  if (!finish_code(p, i, j, (unsigned __int128)Q, p.sta[i], p.stb[j], p.LA[i], p.LB[j], p.slotA[i], p.slotB[j],
                   code))
    return;
  if (p.out) p.out[(size_t)i * p.ldo + j] = code;
  if (F32)
    p.out_f32[(size_t)i * p.ldf + j] =
        bp32_f32_out(code, (p.re ? p.re[i] : 0) + (p.ce ? p.ce[j] : 0), p.bias ? p.bias[j] : 0.0f);
  for (int e = 0; e < p.n_extra; ++e) p.extra_out[e][(size_t)i * p.ldo + p.extra_col0 + j] = code;
}

// The bposit32 of Q * 2^sh + ca + cb (units of 2^lsb_exp; ca, cb 128-bit tail
// corrections): int64 when every part lies in [-2^61, 2^61) (the narrow form's
// usual case: sums of a few tail elements), else the 128-bit rule.
template <int QW>
__device__ __forceinline__ uint32_t finish_with_tails(long long qv, long long qh, int sh, ulonglong2 ca,
                                                      ulonglong2 cb, int lsb_exp) {
  if (QW == 1 && sh <= 61) {
    const long long a = (long long)ca.x, b = (long long)cb.x;
    if ((long long)ca.y == (a >> 63) && (long long)cb.y == (b >> 63) && (a >> 61) == (a >> 63) &&
        (b >> 61) == (b >> 63) && (qv >> (61 - sh)) == (qv >> 63))
      return bp32_from_i64((long long)((unsigned long long)qv << sh) + a + b, lsb_exp);
  }
  const __int128 Q = (__int128)qv + (QW == 2 ? ((__int128)qh << 28) : (__int128)0);
  const unsigned __int128 tot = ((unsigned __int128)Q << sh) + u128(ca) + u128(cb);
  return write_fast_output(tot, lsb_exp + 96, nullptr, nullptr, 0);
}

// Per-column state of a finish item, one entry per column a lane owns: lsb
// base, tail slot, min lsb exponent, exact-window width share (max binade - min
// lsb + ceil log2 K + 3), valid and nonzero flags.
template <int PL>
struct FinishCols {
  int Lj[PL], sj[PL], bx[PL], bw[PL];
  int fe[PL];     // column exponent of the fp32 hand-off (0 without)
  float fb[PL];   // column bias of the fp32 hand-off (0 without)
  bool jv[PL], bz[PL];
};

// Rounds and stores row i of an item from its int64 sums (words qv, qh) and
// row statistics (ra, Li, si).  Whole warp: the tail corrections' loads are
// taken only when some lane of the warp needs them.
template <int PL, int QW>
__device__ __forceinline__ void finish_row_codes(const TcParams &p, const FinishCols<PL> &c, int i, int j0, int lane,
                                           const long long (&qv)[PL], const long long (&qh)[PL], int4 ra, int Li,
                                           int si) {
  uint32_t cd[PL];
  uint32_t slow = 0u, keep = 0u;
#pragma unroll
  for (int q = 0; q < PL; ++q) {
    if (QW == 1) {
      cd[q] = bp32_from_i64(qv[q], Li + c.Lj[q]);
    } else {
      const __int128 Q = (__int128)qv[q] + ((__int128)qh[q] << 28);
      const bool neg = Q < 0;
      const unsigned __int128 m = neg ? (unsigned __int128)0 - (unsigned __int128)Q : (unsigned __int128)Q;
      cd[q] = bp32_from_mag(neg, (uint64_t)(m >> 64), (uint64_t)m, Li + c.Lj[q]);
    }
    const bool plain = si == -1 && c.sj[q] == -1 && ra.z != 0 && c.bz[q] && ra.x + c.bx[q] + 96 >= 0 &&
                       (ra.y - ra.x) + c.bw[q] <= 127;
    if (c.jv[q]) {
      if (plain) keep |= 1u << q;
      else slow |= 1u << q;
    }
  }
  // the others (a tail row or column, a zero row or column, outside the exact
  // window): all their tail corrections are loaded at once, then combined in
  // 128 bits (finish_code's rule)
  if (__any_sync(0xFFFFFFFFu, slow != 0u)) {
    ulonglong2 ca[PL], cb[PL];
#pragma unroll
    for (int q = 0; q < PL; ++q) {
      const bool sb = (slow >> q) & 1u;
      const ulonglong2 z2 = make_ulonglong2(0ull, 0ull);
      ca[q] = (sb && si >= 0) ? p.CA[(size_t)si * p.N + j0 + q * 32 + lane] : z2;
      cb[q] = (sb && c.sj[q] >= 0) ? p.CB[(size_t)c.sj[q] * p.M + i] : z2;
    }
#pragma unroll
    for (int q = 0; q < PL; ++q) {
      if (!((slow >> q) & 1u)) continue;
      if (!(ra.z && c.bz[q])) {
        cd[q] = 0u;
      } else {
        // tc_exact: inside the 128-bit window, no overflowed tail list
        if (ra.x + c.bx[q] + 96 < 0 || (ra.y - ra.x) + c.bw[q] > 127 || si == -2 || c.sj[q] == -2)
          continue;   // left to k_tc_fixup
        cd[q] = finish_with_tails<QW>(qv[q], qh[q], (Li - ra.x) + (c.Lj[q] - c.bx[q]), ca[q], cb[q],
                                      ra.x + c.bx[q]);
      }
      keep |= 1u << q;
    }
  }
  if (p.out) {
    uint32_t *orow = p.out + (size_t)i * p.ldo + j0 + lane;
#pragma unroll
    for (int q = 0; q < PL; ++q)
      if ((keep >> q) & 1u) orow[q * 32] = cd[q];
  }
  for (int e = 0; e < p.n_extra; ++e) {
    uint32_t *erow = p.extra_out[e] + (size_t)i * p.ldo + p.extra_col0 + j0 + lane;
#pragma unroll
    for (int q = 0; q < PL; ++q)
      if ((keep >> q) & 1u) erow[q * 32] = cd[q];
  }
}

template <int PL, int QW>
__device__ __forceinline__ void finish_row_f32(const TcParams &p, const FinishCols<PL> &c, int i, int j0, int lane,
                                           const long long (&qv)[PL], const long long (&qh)[PL], int4 ra, int Li,
                                           int si) {
  uint32_t slow = 0u;
  const int rex = (p.out_f32 && p.re) ? p.re[i] : 0;
  uint32_t *orow = p.out ? p.out + (size_t)i * p.ldo + j0 + lane : nullptr;
  float *frow = p.out_f32 ? p.out_f32 + (size_t)i * p.ldf + j0 + lane : nullptr;
  // one output's stores: its code (output and extra outputs) and fp32 hand-off
  auto put = [&](int q, uint32_t code, float f) {
    if (orow) orow[q * 32] = code;
    if (frow) frow[q * 32] = f;
    for (int e = 0; e < p.n_extra; ++e) p.extra_out[e][(size_t)i * p.ldo + p.extra_col0 + j0 + lane + q * 32] = code;
  };
  // plain outputs (no tail correction, nonzero row and column, inside the
  // exact window) are rounded and stored at once; the others are marked
#pragma unroll
  for (int q = 0; q < PL; ++q) {
    if (!c.jv[q]) continue;
    const bool plain = si == -1 && c.sj[q] == -1 && ra.z != 0 && c.bz[q] && ra.x + c.bx[q] + 96 >= 0 &&
                       (ra.y - ra.x) + c.bw[q] <= 127;
    if (!plain) {
      slow |= 1u << q;
      continue;
    }
    const int L = Li + c.Lj[q];
    uint32_t code = 0u;
    float f = 0.0f;
    if (QW == 1) {
      // the fp32 hand-off straight from the exact sum (bp32_value_i64) when the
      // code is not stored; otherwise from the code
      double v;
      if (frow && !orow && p.n_extra == 0 && bp32_value_i64(qv[q], L, rex + c.fe[q], v)) {
        f = __double2float_rn(v + (double)c.fb[q]);
      } else {
        code = bp32_from_i64(qv[q], L);
        if (frow) f = bp32_f32_out(code, rex + c.fe[q], c.fb[q]);
      }
    } else {
      const __int128 Q = (__int128)qv[q] + ((__int128)qh[q] << 28);
      const bool neg = Q < 0;
      const unsigned __int128 m = neg ? (unsigned __int128)0 - (unsigned __int128)Q : (unsigned __int128)Q;
      code = bp32_from_mag(neg, (uint64_t)(m >> 64), (uint64_t)m, L);
      if (frow) f = bp32_f32_out(code, rex + c.fe[q], c.fb[q]);
    }
    put(q, code, f);
  }
  // the others (a tail row or column, a zero row or column, outside the exact
  // window): all their tail corrections are loaded at once, then combined in
  // 128 bits (finish_code's rule)
  if (__any_sync(0xFFFFFFFFu, slow != 0u)) {
    ulonglong2 ca[PL], cb[PL];
#pragma unroll
    for (int q = 0; q < PL; ++q) {
      const bool sb = (slow >> q) & 1u;
      const ulonglong2 z2 = make_ulonglong2(0ull, 0ull);
      ca[q] = (sb && si >= 0) ? p.CA[(size_t)si * p.N + j0 + q * 32 + lane] : z2;
      cb[q] = (sb && c.sj[q] >= 0) ? p.CB[(size_t)c.sj[q] * p.M + i] : z2;
    }
#pragma unroll
    for (int q = 0; q < PL; ++q) {
      if (!((slow >> q) & 1u)) continue;
      uint32_t code = 0u;
      if (ra.z && c.bz[q]) {
        // tc_exact: inside the 128-bit window, no overflowed tail list
        if (ra.x + c.bx[q] + 96 < 0 || (ra.y - ra.x) + c.bw[q] > 127 || si == -2 || c.sj[q] == -2)
          continue;   // left to k_tc_fixup
        code = finish_with_tails<QW>(qv[q], qh[q], (Li - ra.x) + (c.Lj[q] - c.bx[q]), ca[q], cb[q],
                                     ra.x + c.bx[q]);
      }
      put(q, code, frow ? bp32_f32_out(code, rex + c.fe[q], c.fb[q]) : 0.0f);
    }
  }
}

// Codes only (the kernels without an fp32 output keep this lean form: they
// run beside a GEMM segment at 64 registers) or with the fp32 hand-off.
template <int PL, int QW, bool F32>
__device__ __forceinline__ void finish_row(const TcParams &p, const FinishCols<PL> &c, int i, int j0, int lane,
                                           const long long (&qv)[PL], const long long (&qh)[PL], int4 ra, int Li,
                                           int si) {
  if (F32) finish_row_f32<PL, QW>(p, c, i, j0, lane, qv, qh, ra, Li, si);
  else finish_row_codes<PL, QW>(p, c, i, j0, lane, qv, qh, ra, Li, si);
}

// Blocks per SM the finish kernels are compiled for.  Two (up to 128
// registers) keeps the one-word (bp8) and fp32 variants free of spills: at four
// (64 registers) the bp8 codes-only finish spilled about 600 bytes a thread
// and took 0.53 ms instead of 0.31 beside the headline GEMM's last segment.
// The two-word (bp16) codes-only finish spills little at 64 registers and
// keeps four, so that two of its blocks fit beside a bp16 GEMM segment (at
// two, bp16 8192^3 ran 162.6 TOPS against 168.9).
#ifndef BP_FIN_MINB
#define BP_FIN_MINB 2
#endif
#ifndef BP_FIN_MINB_QW2
#define BP_FIN_MINB_QW2 4
#endif
#ifndef BP_FIN_MINB_F32
#define BP_FIN_MINB_F32 2
#endif
#ifndef BP_FIN_STAGED_MINB_F32
#define BP_FIN_STAGED_MINB_F32 2
#endif
template <int MM, int BN, int QW, bool F32>
__global__ void __launch_bounds__(256, F32 ? BP_FIN_MINB_F32 : (QW == 2 ? BP_FIN_MINB_QW2 : BP_FIN_MINB))
    k_tc_finish(TcParams p, int ntiles, int parts) {
  static_assert(BN % 32 == 0 && MM % 8 == 0 && (QW == 1 || QW == 2), "tile shape");
  constexpr int PL = BN / 32;
  constexpr size_t PT = (size_t)MM * BN;   // words of one plane of a tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl2 = ceil_log2_int(p.K);
  const int4 z4 = make_int4(0, 0, 0, 0);
  // chunk sums stay exact in int64: |word| < 2^60 (bp8) or < 2^53 (bp16 words)
  const bool sum64 = !p.quire && p.split <= (QW == 1 ? 8 : 1024);
  const int rpp = MM / parts;   // rows per item, a multiple of 8
  const long long nitems = (long long)ntiles * parts;
  // After a timed-out wait in any tensor-core GEMM on this device (the error
  // word stays set until bp_device_error reads it), every output is NaR.
  const bool poisoned = *(volatile int *)&g_tc_error != 0;
  for (long long it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int tl = (int)(it / parts), part = (int)(it - (long long)tl * parts);
    const int tile = p.tile0 + tl;
    int tm, tn;
    tile_coords(tile, (p.M + MM - 1) / MM, p.ntn, tm, tn);
    const int j0 = tn * BN;
    if (poisoned) {
      const int rend = min((part + 1) * rpp, p.M - tm * MM);
      for (int r = part * rpp + warp; r < rend; r += 8)
        for (int j = j0 + lane; j < min(j0 + BN, p.N); j += 32) {
          const size_t i = (size_t)(tm * MM + r);
          if (p.out) p.out[i * p.ldo + j] = 0x80000000u;
          if (F32) p.out_f32[i * p.ldf + j] = __uint_as_float(0x7FC00000u);
          for (int e = 0; e < p.n_extra; ++e) p.extra_out[e][i * p.ldo + p.extra_col0 + j] = 0x80000000u;
        }
      continue;
    }
    FinishCols<PL> c;
#pragma unroll
    for (int q = 0; q < PL; ++q) {
      const int j = j0 + q * 32 + lane;
      c.jv[q] = j < p.N;
      const int4 rb = c.jv[q] ? p.stb[j] : z4;
      c.Lj[q] = c.jv[q] ? p.LB[j] : 0;
      c.sj[q] = c.jv[q] ? p.slotB[j] : -1;
      c.bx[q] = rb.x;
      c.bw[q] = (rb.y - rb.x) + cl2 + 3;
      c.bz[q] = rb.z != 0;
      c.fe[q] = (F32 && c.jv[q] && p.ce) ? p.ce[j] : 0;
      c.fb[q] = (F32 && c.jv[q] && p.bias) ? p.bias[j] : 0.0f;
    }
    // rows of this item that exist, relative to the tile; a warp's rows are
    // r0 + 8k
    const int rend = min((part + 1) * rpp, p.M - tm * MM);
    const int r0 = part * rpp + warp;
    const long long *qt = p.qbuf + (size_t)tl * p.split * QW * PT + lane;
    if (!sum64) {
      for (int r = r0; r < rend; r += 8)
#pragma unroll 1
        for (int q = 0; q < PL; ++q) {
          const int j = j0 + q * 32 + lane;
          if (j < p.N) finish_general<QW, F32>(p, qt + (size_t)r * BN + q * 32, PT, tm * MM + r, j);
        }
      continue;
    }
    if (p.split == 1) {
      // software pipeline over the warp's rows: row r + 8's sums and row
      // statistics are in flight while row r is rounded and stored
      long long nq[PL], nh[PL];
      int4 nra = z4;
      int nL = 0, ns = -1;
      auto fetch = [&](int r) {
#pragma unroll
        for (int q = 0; q < PL; ++q) {
          const long long *a = qt + (size_t)r * BN + q * 32;
          nq[q] = c.jv[q] ? __ldcs(a) : 0ll;
          nh[q] = (QW == 2 && c.jv[q]) ? __ldcs(a + PT) : 0ll;
        }
        const int i = tm * MM + r;
        nra = p.sta[i];
        nL = p.LA[i];
        ns = p.slotA[i];
      };
      if (r0 < rend) fetch(r0);
      for (int r = r0; r < rend; r += 8) {
        long long cq[PL], chh[PL];
#pragma unroll
        for (int q = 0; q < PL; ++q) {
          cq[q] = nq[q];
          chh[q] = nh[q];
        }
        const int4 ra = nra;
        const int Li = nL, si = ns;
        if (r + 8 < rend) fetch(r + 8);
        finish_row<PL, QW, F32>(p, c, tm * MM + r, j0, lane, cq, chh, ra, Li, si);
      }
      continue;
    }
    for (int r = r0; r < rend; r += 8) {
      long long cq[PL], chh[PL];
#pragma unroll
      for (int q = 0; q < PL; ++q) cq[q] = chh[q] = 0ll;
      for (int ch = 0; ch < p.split; ++ch) {
#pragma unroll
        for (int q = 0; q < PL; ++q)
          if (c.jv[q]) {
            const long long *a = qt + (size_t)ch * QW * PT + (size_t)r * BN + q * 32;
            cq[q] += __ldcs(a);
            if (QW == 2) chh[q] += __ldcs(a + PT);
          }
      }
      const int i = tm * MM + r;
      finish_row<PL, QW, F32>(p, c, i, j0, lane, cq, chh, p.sta[i], p.LA[i], p.slotA[i]);
    }
  }
  if (p.n_extra) __threadfence_system();
}

// Staged form of the finish for whole-tile launches that have the SMs to
// themselves (the caller's stream, one K chunk, int64 sums, no raw quires):
// thread 0 streams a block's items in chunks of 8 tile rows -- one row per
// warp, QW planes of 8 x BN int64 sums, contiguous in the tile-compact buffer
// -- with bulk copies into a ring of kFinStages shared-memory buffers, each
// with its own mbarrier, so several chunks per block are in flight while the
// warps round the previous ones from shared memory (the per-thread loads of
// k_tc_finish left the kernel stalled on their latency at a third of HBM
// bandwidth).  A chunk's buffer is refilled after a block barrier that ends
// its use.  Waits are bounded: a timeout records code 16 in g_tc_error, and
// the block stops after the barrier at which it learns of it.
constexpr int kFinStages = 4;

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int MM, int BN, int QW>
size_t finish_staged_smem() {
  return (size_t)kFinStages * QW * 8 * BN * sizeof(long long) + kFinStages * sizeof(uint64_t);
}

template <int MM, int BN, int QW, bool F32>
__global__ void __launch_bounds__(256, F32 ? BP_FIN_STAGED_MINB_F32 : (QW == 2 ? BP_FIN_MINB_QW2 : BP_FIN_MINB))
    k_tc_finish_staged(TcParams p, int ntiles, int parts) {
  static_assert(BN % 32 == 0 && MM % 8 == 0 && (QW == 1 || QW == 2), "tile shape");
  constexpr int PL = BN / 32;
  constexpr size_t PT = (size_t)MM * BN;              // words of one plane of a tile
  constexpr uint32_t CHUNK = 8u * BN * 8u;            // bytes of one plane of a chunk (16-byte multiple)
  extern __shared__ __align__(16) uint8_t fsm[];
  long long *buf = (long long *)fsm;                  // [kFinStages][QW][8][BN]
  uint64_t *bar = (uint64_t *)(fsm + (size_t)kFinStages * QW * CHUNK);
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl2 = ceil_log2_int(p.K);
  const int4 z4 = make_int4(0, 0, 0, 0);
  const int rpp = MM / parts, cpi = rpp / 8;          // rows and chunks per item
  const long long nitems = (long long)ntiles * parts;
  const long long mine = (long long)blockIdx.x < nitems ? (nitems - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const long long total = mine * cpi;
  if (*(volatile int *)&g_tc_error != 0) {
    // a tensor-core GEMM on this device gave up on a bounded wait: NaR everywhere
    for (long long it = blockIdx.x; it < nitems; it += gridDim.x) {
      const int tl = (int)(it / parts), part = (int)(it - (long long)tl * parts);
      int tm, tn;
      tile_coords(p.tile0 + tl, (p.M + MM - 1) / MM, p.ntn, tm, tn);
      const int rend = min((part + 1) * rpp, p.M - tm * MM);
      for (int r = part * rpp + warp; r < rend; r += 8)
        for (int j = tn * BN + lane; j < min(tn * BN + BN, p.N); j += 32) {
          const size_t i = (size_t)(tm * MM + r);
          if (p.out) p.out[i * p.ldo + j] = 0x80000000u;
          if (F32) p.out_f32[i * p.ldf + j] = __uint_as_float(0x7FC00000u);
          for (int e = 0; e < p.n_extra; ++e) p.extra_out[e][i * p.ldo + p.extra_col0 + j] = 0x80000000u;
        }
    }
    return;
  }
  // Chunk g of this block is chunk g % cpi of its item g / cpi; both are
  // walked with counters (a 64-bit division per chunk cost more than the
  // chunk's rounding).  Thread 0's issue cursor: item ii, chunk ic, the
  // item's source rows.
  long long ii = 0;
  int ic = 0;
  const long long *isrc = nullptr;
  auto issue = [&](long long g) {   // thread 0: bulk copies of the next chunk (g) into buffer g % kFinStages
    if (ic == 0) {
      const long long it = blockIdx.x + ii * gridDim.x;
      const int tl = (int)(it / parts), part = (int)(it - (long long)tl * parts);
      isrc = p.qbuf + (size_t)tl * QW * PT + (size_t)(part * rpp) * BN;
    }
    const long long *src = isrc + (size_t)(8 * ic) * BN;
    const int st = (int)(g % kFinStages);
    mbar_expect_tx(&bar[st], QW * CHUNK);
#pragma unroll
    for (int w = 0; w < QW; ++w) bulk_g2s(buf + ((size_t)st * QW + w) * 8 * BN, src + w * PT, CHUNK, &bar[st]);
    if (++ic == cpi) {
      ic = 0;
      ++ii;
    }
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < kFinStages; ++st) mbar_init(&bar[st], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (long long g = 0; g < total && g < kFinStages; ++g) issue(g);
  }
  __syncthreads();
  FinishCols<PL> c;
  long long item = 0;
  int ci = 0;
  int tm = 0, tn = 0, j0 = 0, part = 0, rend = 0;
  for (long long g = 0; g < total; ++g) {
    if (ci == 0) {   // columns of the new item, loaded once
      const long long it = blockIdx.x + item * gridDim.x;
      const int tl = (int)(it / parts);
      part = (int)(it - (long long)tl * parts);
      tile_coords(p.tile0 + tl, (p.M + MM - 1) / MM, p.ntn, tm, tn);
      j0 = tn * BN;
      rend = min((part + 1) * rpp, p.M - tm * MM);
#pragma unroll
      for (int q = 0; q < PL; ++q) {
        const int j = j0 + q * 32 + lane;
        c.jv[q] = j < p.N;
        const int4 rb = c.jv[q] ? p.stb[j] : z4;
        c.Lj[q] = c.jv[q] ? p.LB[j] : 0;
        c.sj[q] = c.jv[q] ? p.slotB[j] : -1;
        c.bx[q] = rb.x;
        c.bw[q] = (rb.y - rb.x) + cl2 + 3;
        c.bz[q] = rb.z != 0;
        c.fe[q] = (F32 && c.jv[q] && p.ce) ? p.ce[j] : 0;
        c.fb[q] = (F32 && c.jv[q] && p.bias) ? p.bias[j] : 0.0f;
      }
    }
    const int st = (int)(g % kFinStages);
    const uint32_t par = (uint32_t)(g / kFinStages) & 1u;
    bool ok = true;
    {
      const long long t0 = clock64();
      while (!mbar_try_wait(&bar[st], par)) {
        if (clock64() - t0 > WAIT_LIMIT) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) {
      atomicOr(&g_tc_error, 16);
      s_abort = 1;
    }
    const int r = part * rpp + 8 * ci + warp;
    if (ok && r < rend) {
      const long long *row = buf + (size_t)st * QW * 8 * BN + (size_t)warp * BN + lane;
      long long qv[PL], qh[PL];
#pragma unroll
      for (int q = 0; q < PL; ++q) {
        qv[q] = c.jv[q] ? row[q * 32] : 0ll;
        qh[q] = (QW == 2 && c.jv[q]) ? row[8 * BN + q * 32] : 0ll;
      }
      const int i = tm * MM + r;
      finish_row<PL, QW, F32>(p, c, i, j0, lane, qv, qh, p.sta[i], p.LA[i], p.slotA[i]);
    }
    __syncthreads();   // every warp is done with buffer st
    if (s_abort) break;
    if (threadIdx.x == 0 && g + kFinStages < total) issue(g + kFinStages);
    if (++ci == cpi) {
      ci = 0;
      ++item;
    }
  }
  if (p.n_extra) __threadfence_system();
}

// ----------------------------------------------------------- digit planes ---
template <int FMT>
__device__ __forceinline__ ElemME decode_scaled(uint32_t c, const int32_t *s, int row, int k, int G, int group) {
  ElemME r;
  if (FMT == 8) posit_to_me<8, 2>(c, r.m, r.e);
  else posit_to_me<16, 3>(c, r.m, r.e);
  if (s && r.m) r.e += s[(size_t)row * G + k / group];
  return r;
}

template <int FMT>
__device__ __forceinline__ uint32_t load_code(const void *codes, size_t idx) {
  return FMT == 8 ? (uint32_t)((const uint8_t *)codes)[idx] : (uint32_t)((const uint16_t *)codes)[idx];
}

// 16 bytes of codes: 16 bp8 or 8 bp16 codes into c[].
template <int FMT>
__device__ __forceinline__ void load_codes16(const void *codes, size_t idx, uint32_t *c) {
  uint4 w = *(const uint4 *)((const uint8_t *)codes + idx * (FMT / 8));
  uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  if (FMT == 8) {
#pragma unroll
    for (int q = 0; q < 16; ++q) c[q] = (ws[q >> 2] >> (8 * (q & 3))) & 0xFFu;
  } else {
#pragma unroll
    for (int q = 0; q < 8; ++q) c[q] = (ws[q >> 1] >> (16 * (q & 1))) & 0xFFFFu;
  }
}

// Block-wide min of lo and max of hi and nz in one exchange (one barrier).  The
// caller keeps a barrier between two uses of `red` (the next row's exchange
// starts only after this row's later barriers).
__device__ __forceinline__ void block_minmax(int &lo, int &hi, int &nz, int4 *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
    nz |= __shfl_xor_sync(0xFFFFFFFFu, nz, o);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_int4(lo, hi, nz, 0);
  __syncthreads();
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    const int4 v = red[w];
    lo = min(lo, v.x);
    hi = max(hi, v.y);
    nz |= v.z;
  }
}

// Each byte of the result: 0xFF where bit 7 of that byte of a is set, else 0
// (prmt's sign-replicating selector nibbles 8..B).
__device__ __forceinline__ uint32_t byte_signs(uint32_t a) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(0u), "r"(0xBA98u));
  return d;
}

// Two 16-bit lanes per register: native unsigned min / max (sm_90 and later).
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// bp8 decode table entry: lsb exponent, binade and signed mantissa packed in
// 10 + 10 + 12 bits (bp8: |lsb|, |binade| <= 24, |mantissa| <= 15).
__device__ __forceinline__ uint32_t dec_pack(int lsb, int hb, int m) {
  return (uint32_t)(lsb + 512) | ((uint32_t)(hb + 512) << 10) | ((uint32_t)(m + 2048) << 20);
}
__device__ __forceinline__ int dec_lsb(uint32_t t) { return (int)(t & 1023u) - 512; }
__device__ __forceinline__ int dec_hb(uint32_t t) { return (int)((t >> 10) & 1023u) - 512; }
__device__ __forceinline__ int dec_m(uint32_t t) { return (int)(t >> 20) - 2048; }

// Decoded element: lsb exponent (group scale folded in) and signed mantissa.
template <int FMT>
__device__ __forceinline__ ElemME prep_decode(uint32_t c, const uint32_t *s_dec) {
  ElemME x;
  if (FMT == 8) {
    uint32_t t = s_dec[c];
    x.m = dec_m(t);
    x.e = dec_lsb(t);
  } else {
    posit_to_me<16, 3>(c, x.m, x.e);
  }
  return x;
}

// One block per row: statistics, main base L, S digit planes, tail list and
// correction slot.  Pass 2 re-reads the row, which is still in L2.  bp8 codes
// are decoded through a 256-entry table; for unscaled bp8 rows pass 2 also
// uses a per-row table of each code's packed digits (bit 31 marks a tail).
// One operand of a prep launch.
struct PrepOp {
  const void *codes;
  int rows;
  const int32_t *sc;
  int4 *stats;
  int8_t *planes;
  int *Lr, *slot;
  int4 *seg;
  int *tails;
  int cap;
  TcCounters *ctr;
};

template <int FMT, int S>
__global__ void __launch_bounds__(256, 5) k_tc_prep(const PrepOp opA, const PrepOp opB, int K, int Kp, int G,
                                                 int group, int pool_cap) {
  constexpr int SPAN = Cfg<S>::SPAN;
  constexpr int DB = Cfg<S>::DB, HALF = Cfg<S>::HALF, DMASK = (1 << DB) - 1;   // digit base 2^DB
  constexpr int EPT = FMT == 8 ? 16 : 8;   // elements per 16-byte load
  constexpr bool LUT_DIGITS = FMT == 8 && S <= 4;
  __shared__ int s_tail[TAILCAP];
  __shared__ uint32_t s_dec[FMT == 8 ? 256 : 1];  // packed lsb | binade | mantissa (dec_* below)
  __shared__ uint32_t s_dig[FMT == 8 ? 256 : 1];
  __shared__ int4 red[8];
  __shared__ int s_nt, s_off, s_slot;
  if (FMT == 8) {
    for (int c = threadIdx.x; c < 256; c += blockDim.x) {
      int m, e;
      posit_to_me<8, 2>((uint32_t)c, m, e);
      int hb = m ? e + 31 - __clz(m < 0 ? -m : m) : 0;
      s_dec[c] = dec_pack(e, hb, m);
    }
    __syncthreads();
  }
  // rows of A, then rows of B: both operands in one launch (block-uniform choice)
  for (int rr = blockIdx.x; rr < opA.rows + opB.rows; rr += gridDim.x) {
    const bool second = rr >= opA.rows;
    const int r = second ? rr - opA.rows : rr;
    const void *__restrict__ codes = second ? opB.codes : opA.codes;
    const int rows = second ? opB.rows : opA.rows;
    const int32_t *__restrict__ sc = second ? opB.sc : opA.sc;
    int4 *__restrict__ stats = second ? opB.stats : opA.stats;
    int8_t *__restrict__ planes = second ? opB.planes : opA.planes;
    int *__restrict__ Lr = second ? opB.Lr : opA.Lr;
    int *__restrict__ slot = second ? opB.slot : opA.slot;
    int4 *__restrict__ seg = second ? opB.seg : opA.seg;
    int *__restrict__ tails = second ? opB.tails : opA.tails;
    const int cap = second ? opB.cap : opA.cap;
    TcCounters *__restrict__ ctr = second ? opB.ctr : opA.ctr;
    const size_t plane = (size_t)rows * Kp;
    const bool vec = (K % EPT) == 0 && (((uintptr_t)codes) & 15u) == 0;
    const size_t rb = (size_t)r * K;
    // pass 1: statistics.  A posit's lsb exponent and binade are both
    // non-decreasing in its magnitude, so the row's min lsb and max binade are
    // those of its smallest and largest nonzero code magnitude (per group
    // chunk when group scales are present).
    int lo = 0x3FFFFFFF, hi = -0x3FFFFFFF, nz = 0;
    const bool chunk_groups = sc != nullptr && (group % EPT) == 0;
    if (FMT == 8 && sc == nullptr && vec) {
      // unscaled bp8: the code magnitudes |c| = min(c, 256 - c) in two 16-bit
      // lanes per register (0 for zero, 128 only for NaR), a running max of
      // |c| and a running min of |c| - 1 (zero -> 0x7FFF), seven instructions
      // per two codes.  A NaR makes the max 128: the rare thread that saw one
      // redoes its span code by code, leaving out zero and NaR.  Decoded once
      // at the end.
      // Each thread's next 16 codes are loaded one step ahead.
      uint32_t mnw = 0x7FFF7FFFu, mxw = 0u;
      const int step = blockDim.x * 16;
      uint4 nxt = make_uint4(0u, 0u, 0u, 0u);
      if (threadIdx.x * 16 < K) nxt = *(const uint4 *)((const uint8_t *)codes + rb + threadIdx.x * 16);
      for (int k0 = threadIdx.x * 16; k0 < K; k0 += step) {
        const uint4 cw = nxt;
        if (k0 + step < K) nxt = *(const uint4 *)((const uint8_t *)codes + rb + k0 + step);
        const uint32_t ws[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t x = __byte_perm(ws[q >> 1], 0u, (q & 1) ? 0x4341u : 0x4240u);   // two codes, 16-bit lanes
          const uint32_t mag = min_u16x2(x, 0x01000100u - x);
          mxw = max_u16x2(mxw, mag);
          mnw = min_u16x2(mnw, (mag + 0x7FFF7FFFu) & 0x7FFF7FFFu);   // no carry between the lanes: |c| <= 128
        }
      }
      uint32_t mn = min(mnw & 0xFFFFu, mnw >> 16) + 1u;
      uint32_t mx = max(mxw & 0xFFFFu, mxw >> 16);
      if (mx == 128u) {
        mn = 0xFFu;
        mx = 0u;
        for (int k0 = threadIdx.x * 16; k0 < K; k0 += blockDim.x * 16)
          for (int q = 0; q < 16; ++q) {
            const uint32_t c = ((const uint8_t *)codes)[rb + k0 + q];
            if (c & 0x7Fu) {
              const uint32_t mag = (c & 0x80u) ? 256u - c : c;
              mn = min(mn, mag);
              mx = max(mx, mag);
            }
          }
      }
      if (mx) {
        lo = dec_lsb(s_dec[mn]);
        hi = dec_hb(s_dec[mx]);
        nz = 1;
      }
    } else
    for (int k0 = threadIdx.x * EPT; k0 < K; k0 += blockDim.x * EPT) {
      uint32_t c[EPT];
      if (vec) {
        load_codes16<FMT>(codes, rb + k0, c);
      } else {
#pragma unroll
        for (int q = 0; q < EPT; ++q) c[q] = k0 + q < K ? load_code<FMT>(codes, rb + k0 + q) : 0u;
      }
      if (sc == nullptr || chunk_groups) {
        uint32_t mn = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const uint32_t sb = FMT == 8 ? 0x80u : 0x8000u;
          uint32_t mag = (c[q] & sb) ? (2u * sb - c[q]) : c[q];
          bool v = (c[q] & (sb - 1u)) != 0u;          // not zero, not NaR
          mn = v ? min(mn, mag) : mn;
          mx = v ? max(mx, mag) : mx;
        }
        if (mx) {
          int sc_ = sc ? sc[(size_t)r * G + k0 / group] : 0;
          int l, h;
          if (FMT == 8) {
            l = dec_lsb(s_dec[mn]);
            h = dec_hb(s_dec[mx]);
          } else {
            Dec d0 = decode_posit<16, 3>(mn), d1 = decode_posit<16, 3>(mx);
            l = d0.scale - d0.fw;
            h = d1.scale;
          }
          lo = min(lo, l + sc_);
          hi = max(hi, h + sc_);
          nz = 1;
        }
      } else {
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          int l, h;
          if (FMT == 8) {
            uint32_t t = s_dec[c[q]];
            if (!dec_m(t)) continue;
            l = dec_lsb(t);
            h = dec_hb(t);
          } else {
            Dec d = decode_posit<16, 3>(c[q]);
            if (d.kind != 0) continue;
            l = d.scale - d.fw;
            h = d.scale;
          }
          int sc_ = sc[(size_t)r * G + (k0 + q) / group];
          lo = min(lo, l + sc_);
          hi = max(hi, h + sc_);
          nz = 1;
        }
      }
    }
    block_minmax(lo, hi, nz, red);
    const int L = nz ? max(lo, hi - (SPAN - 1)) : 0;
    if (threadIdx.x == 0) {
      stats[r] = make_int4(nz ? lo : 0, nz ? hi : 0, nz, 0);
      Lr[r] = L;
      s_nt = 0;
      if (nz) {
        atomicMax(&ctr->v[2], BIG - lo);
        atomicMax(&ctr->v[3], hi - lo);
        atomicMax(&ctr->v[5], 1);
      }
    }
    const bool lut = LUT_DIGITS && sc == nullptr;
    if (lut) {
      for (int cc = threadIdx.x; cc < 256; cc += blockDim.x) {
        uint32_t t = s_dec[cc];
        uint32_t v = 0u;
        if (dec_m(t)) {
          if (dec_lsb(t) < L) {
            v = 0x80000000u;
          } else {
            int x = dec_m(t) * (1 << (dec_lsb(t) - L));
#pragma unroll
            for (int s = 0; s < S - 1; ++s) {
              int dg = ((x + HALF) & DMASK) - HALF;
              v |= ((uint32_t)(uint8_t)dg) << (8 * s);
              x = (x - dg) >> DB;
            }
            v |= ((uint32_t)(uint8_t)x) << (8 * (S - 1));
          }
        }
        s_dig[cc] = v;
      }
    }
    __syncthreads();
    // pass 2: digit planes and tail list
    int8_t *row = planes + (size_t)r * Kp;
    if (lut && vec) {
      // unscaled bp8: every code's S digits come packed in one table word
      // (bit 31 = tail); plane words are assembled with byte permutes
      // last read of these codes (each thread's next 16 loaded one step
      // ahead); the plane stores below stream past L2 (evict-first) so that
      // this second pass finds its row still there
      const int step = blockDim.x * 16;
      uint4 nxt = make_uint4(0u, 0u, 0u, 0u);
      if (threadIdx.x * 16 < K) nxt = __ldcs((const uint4 *)((const uint8_t *)codes + rb + threadIdx.x * 16));
      for (int k0 = threadIdx.x * 16; k0 < Kp; k0 += step) {
        uint32_t v[16];
        uint32_t any = 0u;
        const uint4 cw = nxt;
        if (k0 + step < K) nxt = __ldcs((const uint4 *)((const uint8_t *)codes + rb + k0 + step));
        if (k0 < K) {
          uint32_t ws[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            v[q] = s_dig[(ws[q >> 2] >> (8 * (q & 3))) & 0xFFu];
            any |= v[q];
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = 0u;
        }
        if (any & 0x80000000u) {
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (v[q] & 0x80000000u) {
              int pos = atomicAdd(&s_nt, 1);
              if (pos < TAILCAP) s_tail[pos] = k0 + q;
            }
        }
        if (S == 3) {
          // 4 x 3 byte transpose per 4 codes: 7 permutes for the three plane words
          uint32_t wd[3][4];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t a01 = __byte_perm(v[4 * g], v[4 * g + 1], 0x5140);      // d0 d0' d1 d1'
            const uint32_t a23 = __byte_perm(v[4 * g + 2], v[4 * g + 3], 0x5140);
            const uint32_t b01 = __byte_perm(v[4 * g], v[4 * g + 1], 0x0062);      // d2 d2'
            const uint32_t b23 = __byte_perm(v[4 * g + 2], v[4 * g + 3], 0x0062);
            wd[0][g] = __byte_perm(a01, a23, 0x5410);
            wd[1][g] = __byte_perm(a01, a23, 0x7632);
            wd[2][g] = __byte_perm(b01, b23, 0x5410);
          }
#pragma unroll
          for (int sd = 0; sd < 3; ++sd)
            __stcs((uint4 *)(row + sd * plane + k0), make_uint4(wd[sd][0], wd[sd][1], wd[sd][2], wd[sd][3]));
        } else if (S == 2) {
          // 4 x 2 byte transpose per 4 codes: 4 permutes for the two plane words
          uint32_t wd[2][4];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t a01 = __byte_perm(v[4 * g], v[4 * g + 1], 0x5140);      // d0 d0' d1 d1'
            const uint32_t a23 = __byte_perm(v[4 * g + 2], v[4 * g + 3], 0x5140);
            wd[0][g] = __byte_perm(a01, a23, 0x5410);
            wd[1][g] = __byte_perm(a01, a23, 0x7632);
          }
#pragma unroll
          for (int sd = 0; sd < 2; ++sd)
            __stcs((uint4 *)(row + sd * plane + k0), make_uint4(wd[sd][0], wd[sd][1], wd[sd][2], wd[sd][3]));
        } else {
#pragma unroll
          for (int sd = 0; sd < S; ++sd) {
            const uint32_t sel = (uint32_t)sd | ((uint32_t)(4 + sd) << 4);
            uint32_t wd[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint32_t lo2 = __byte_perm(v[4 * g], v[4 * g + 1], sel);
              uint32_t hi2 = __byte_perm(v[4 * g + 2], v[4 * g + 3], sel);
              wd[g] = __byte_perm(lo2, hi2, 0x5410);
            }
            __stcs((uint4 *)(row + sd * plane + k0), make_uint4(wd[0], wd[1], wd[2], wd[3]));
          }
        }
      }
    } else {
      for (int k0 = threadIdx.x * EPT; k0 < Kp; k0 += blockDim.x * EPT) {
        uint32_t c[EPT];
        if (vec && k0 < K) {
          load_codes16<FMT>(codes, rb + k0, c);
        } else {
#pragma unroll
          for (int q = 0; q < EPT; ++q) c[q] = k0 + q < K ? load_code<FMT>(codes, rb + k0 + q) : 0u;
        }
        uint32_t w[S][EPT / 4];
#pragma unroll
        for (int sd = 0; sd < S; ++sd)
#pragma unroll
          for (int q = 0; q < EPT / 4; ++q) w[sd][q] = 0u;
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
          const int k = k0 + q;
          if (lut) {
            uint32_t v = s_dig[c[q]];
            if (v & 0x80000000u) {
              int pos = atomicAdd(&s_nt, 1);
              if (pos < TAILCAP) s_tail[pos] = k;
              continue;
            }
#pragma unroll
            for (int sd = 0; sd < S; ++sd) w[sd][q >> 2] |= ((v >> (8 * sd)) & 0xFFu) << (8 * (q & 3));
            continue;
          }
          ElemME x = prep_decode<FMT>(c[q], s_dec);
          if (!x.m || k >= K) continue;
          if (sc) x.e += sc[(size_t)r * G + k / group];
          if (x.e < L) {
            int pos = atomicAdd(&s_nt, 1);
            if (pos < TAILCAP) s_tail[pos] = k;
            continue;
          }
          int t = x.m * (1 << (x.e - L));
#pragma unroll
          for (int sd = 0; sd < S - 1; ++sd) {
            int dg = ((t + HALF) & DMASK) - HALF;
            w[sd][q >> 2] |= ((uint32_t)(uint8_t)dg) << (8 * (q & 3));
            t = (t - dg) >> DB;
          }
          w[S - 1][q >> 2] |= ((uint32_t)(uint8_t)t) << (8 * (q & 3));
        }
#pragma unroll
        for (int sd = 0; sd < S; ++sd) {
          if (EPT == 16) *(uint4 *)(row + sd * plane + k0) = make_uint4(w[sd][0], w[sd][1], w[sd][2], w[sd][3]);
          else *(uint2 *)(row + sd * plane + k0) = make_uint2(w[sd][0], w[sd][1]);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const int nt = s_nt;
      int sl = -1, off = 0;
      if (nt) {
        sl = atomicAdd(&ctr->v[0], 1);
        bool fits = nt <= TAILCAP;
        if (fits) {
          off = atomicAdd(&ctr->v[1], nt);
          fits = off + nt <= pool_cap;
        }
        if (sl < cap) seg[sl] = make_int4(off, fits ? nt : 0, r, 0);
        if (sl >= cap || !fits) {
          sl = -2;
          atomicMax(&ctr->v[4], 1);
        }
      }
      slot[r] = sl;
      s_slot = sl;
      s_off = off;
    }
    __syncthreads();
    if (s_slot >= 0)
      for (int t = threadIdx.x; t < s_nt; t += blockDim.x) tails[s_off + t] = s_tail[t];
    // no barrier here: the next row touches s_nt, s_tail and the tables only
    // after the barrier of its statistics exchange
  }
}

// ------------------------------------------------------- tail correction ---
// For each listed tail row x of operand X (slot s), over all rows y of Y:
//   C[s][y] = sum over its tail elements (x, k):  v(X[x,k]) * v(Y[y,k])
// exactly, in units of 2^(la_x + la_y).  When YL is given, Y's own tail
// elements (lsb below YL[y]) are skipped (they are counted from Y's side).
// One side of the correction launch.  blockIdx.z selects the side; each side
// runs on its own gx x gy corner of the launch's grid (the rest of that
// side's blocks exit), so both sides are one launch.
struct CorrSide {
  const void *X, *Y;
  int Yrows;
  const int32_t *xs, *ys;
  const int4 *xst, *yst;
  const int *YL;
  const int4 *seg;
  const int *tails;
  const TcCounters *ctr;
  int cap;
  ulonglong2 *Cout;
  int gx, gy;
};

template <int FMT>
__global__ void __launch_bounds__(256) k_tc_corr(const CorrSide s0, const CorrSide s1, int K, int G, int group) {
  const bool second = blockIdx.z != 0;
  const int gx = second ? s1.gx : s0.gx, gy = second ? s1.gy : s0.gy;
  if ((int)blockIdx.x >= gx || (int)blockIdx.y >= gy) return;
  const void *__restrict__ X = second ? s1.X : s0.X;
  const void *__restrict__ Y = second ? s1.Y : s0.Y;
  const int Yrows = second ? s1.Yrows : s0.Yrows;
  const int32_t *__restrict__ xs = second ? s1.xs : s0.xs;
  const int32_t *__restrict__ ys = second ? s1.ys : s0.ys;
  const int4 *__restrict__ xst = second ? s1.xst : s0.xst;
  const int4 *__restrict__ yst = second ? s1.yst : s0.yst;
  const int *__restrict__ YL = second ? s1.YL : s0.YL;
  const int4 *__restrict__ seg = second ? s1.seg : s0.seg;
  const int *__restrict__ tails = second ? s1.tails : s0.tails;
  const TcCounters *__restrict__ ctr = second ? s1.ctr : s0.ctr;
  ulonglong2 *__restrict__ Cout = second ? s1.Cout : s0.Cout;
  const int nslots = min(ctr->v[0], second ? s1.cap : s0.cap);
  for (int sl = blockIdx.x; sl < nslots; sl += gx) {
    const int4 sg = seg[sl];
    const int x = sg.z;
    const int la_x = xst[x].x;
    for (int y0 = blockIdx.y * 256; y0 < Yrows; y0 += gy * 256) {
      const int y = y0 + threadIdx.x;
      if (y >= Yrows) continue;
      const int la_y = yst[y].x;
      const int Ly = YL ? YL[y] : -0x3FFFFFFF;
      unsigned __int128 acc = 0;
      for (int t = 0; t < sg.y; ++t) {
        const int k = tails[sg.x + t];
        ElemME e = decode_scaled<FMT>(load_code<FMT>(X, (size_t)x * K + k), xs, x, k, G, group);
        ElemME f = decode_scaled<FMT>(load_code<FMT>(Y, (size_t)y * K + k), ys, y, k, G, group);
        if (!f.m || f.e < Ly) continue;
        long long P = (long long)e.m * f.m;
        int sh = e.e + f.e - (la_x + la_y);
        sh = min(max(sh, 0), 127);
        acc += (unsigned __int128)(__int128)P << sh;
      }
      Cout[(size_t)sl * Yrows + y] = make_ulonglong2((unsigned long long)acc, (unsigned long long)(acc >> 64));
    }
  }
}

// K-major copies for the narrow form's corrections, decoded: codes [rows][K]
// (bp8) -> [K][2 ldt] bytes (ldt = rows rounded up to 16, padding columns
// zero) holding two byte planes: M, the signed mantissa m (value = m 2^lsb,
// |m| <= 15), and E, the lsb exponent above the row's minimum, lsb - la_r
// (0 .. hb_r - la_r, below 64 for bp8).  Row k is cut into blocks of
// kCorrPass (512) columns, the last one narrower (w = min(512, ldt - 512 b)
// for block b); block b sits at byte 1024 b of the row, its w M bytes first
// and its w E bytes after them.  A correction pass over one block of a tail
// element's column is then one contiguous copy, and needs no table.  With `Lr`
// (the rows' main bases) every element whose lsb lies below its row's base --
// a listed tail element -- is written as m = 0: the copy holds the main part.
// Zero and NaR are m = 0.
// Blocks stride over tiles of 64 rows x 128 columns: thread t loads 8 bytes
// of each of 4 rows, transposes the two 4 x 4 blocks in registers (byte
// permutes) and parks the raw code words in shared memory (local row kk's
// word slots rotated by kk / 8, so a warp's stores spread over the banks);
// then four threads take the 64 codes of one output row, each decoding its 16
// through a table with one copy per lane (entry (code, lane) in the 32-bit
// word 32 (code >> 1) + lane, half-word code & 1: every lane reads its own
// bank), and store 16 bytes of each plane.  Decoding after the transpose
// moves one byte per code through the staging instead of two; the decode
// before it used a 16-copy table with up to 4-way bank conflicts.  Each thread
// issues a tile's loads two tiles before it works on it (a copy with one
// tile's loads in flight per thread was bound by their latency).  25 KB of
// shared memory lets two blocks sit beside a narrow-form GEMM CTA.  The
// blocks of the first column of tiles also record, per 64 rows, the widest
// row range hb - la (hr64, zeroed by the caller).  kKmajSmem bytes of
// dynamic shared memory.
constexpr int kKmajK = 128;
constexpr size_t kKmajTable = 128 * 32 * 4;   // 256 codes x 32 lanes, 16-bit entries
constexpr size_t kKmajSmem = (size_t)kKmajK * 17 * 4 + kKmajTable;

// One tile's global loads, issued two tiles ahead of their use: the thread's
// 8 bytes of each of its 4 rows, and (threads < 64) the tile row's minimum lsb
// and main base.  A tile past the end loads nothing.
struct KmajFetch {
  uint2 w[4];
  int la, L;
};

__device__ __forceinline__ void kmaj_fetch(long long tile, long long ntiles, int tk, const uint8_t *__restrict__ src,
                                           int rows, int K, bool vec, const int4 *__restrict__ st,
                                           const int *__restrict__ Lr, int t, int br, int bc, KmajFetch &f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) f.w[i] = make_uint2(0u, 0u);
  f.la = 0;
  f.L = -0x3FFFFFFF;
  if (tile >= ntiles) return;
  const int k0 = (int)(tile % tk) * kKmajK, r0 = (int)(tile / tk) * 64;
  if (t < 64 && r0 + t < rows) {
    f.la = __ldg(&st[r0 + t].x);
    if (Lr) f.L = __ldg(&Lr[r0 + t]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + 4 * br + i, k = k0 + 8 * bc;
    if (r < rows) {
      const uint8_t *row = src + (size_t)r * K;
      if (vec && k + 8 <= K) {
        f.w[i] = __ldcs((const uint2 *)(row + k));
      } else {
        uint32_t b[2] = {0u, 0u};
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (k + q < K) b[q >> 2] |= (uint32_t)row[k + q] << (8 * (q & 3));
        f.w[i] = make_uint2(b[0], b[1]);
      }
    }
  }
}

// The (lsb + 64) << 8 | (uint8) m entries of the four codes in word v (bytes
// in row order), read from this lane's copy of the table; byte address of
// entry (code, lane): 128 (code >> 1) + 4 lane + 2 (code & 1).
__device__ __forceinline__ void kmaj_decode4(uint32_t v, const uint8_t *s_tab, uint32_t lane4, uint32_t &mw,
                                             uint32_t &lw) {
  uint32_t d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t b = (v >> (8 * i)) & 0xFFu;
    d[i] = *(const uint16_t *)(s_tab + (((b >> 1) << 7) | lane4 | ((b & 1u) << 1)));
  }
  const uint32_t lo = d[0] | (d[1] << 16), hi = d[2] | (d[3] << 16);
  mw = __byte_perm(lo, hi, 0x6420);
  lw = __byte_perm(lo, hi, 0x7531);
}

// One tile from its fetched loads: transpose the codes through shared memory,
// decode, store the two planes' 128 output rows of 64 bytes.
__device__ __forceinline__ void kmaj_tile(long long tile, int tk, int rows, int K, uint8_t *__restrict__ dme,
                                          int ldt, const int4 *__restrict__ st,
                                          int *__restrict__ hr64, int t, int br, int bc, const KmajFetch &f,
                                          uint32_t (*tc)[17], const uint8_t *s_tab, uint8_t *s_la4,
                                          uint8_t *s_L4) {
  const int k0 = (int)(tile % tk) * kKmajK, r0 = (int)(tile / tk) * 64;
  __syncthreads();   // the previous tile's rows and staging are no longer read
  if (t < 64) {
    // per tile row: la + 64 and the base L + 64 clamped to 1 .. 127 (1 keeps
    // every nonzero element: a row without a base, B's whole copy), one byte
    // each, so that word w holds rows 4w .. 4w + 3
    s_la4[t] = (uint8_t)(f.la + 64);
    s_L4[t] = (uint8_t)min(max(f.L + 64, 1), 127);
    // the widest row range (hb - la) of these 64 rows, once per row block: it
    // bounds the E plane here, for the corrections' choice of arithmetic
    if (k0 == 0) {
      int h = r0 + t < rows ? __ldg(&st[r0 + t].y) - f.la : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) h = max(h, __shfl_xor_sync(0xFFFFFFFFu, h, o));
      if ((t & 31) == 0) atomicMax(&hr64[r0 / 64], h);
    }
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {   // columns 4g .. 4g + 3 of the thread's 8
    const uint32_t r0w = g ? f.w[0].y : f.w[0].x, r1w = g ? f.w[1].y : f.w[1].x;
    const uint32_t r2w = g ? f.w[2].y : f.w[2].x, r3w = g ? f.w[3].y : f.w[3].x;
    // column q: byte q of each row word (bytes in row order)
    const uint32_t a01 = __byte_perm(r0w, r1w, 0x5140), a23 = __byte_perm(r2w, r3w, 0x5140);
    const uint32_t b01 = __byte_perm(r0w, r1w, 0x7362), b23 = __byte_perm(r2w, r3w, 0x7362);
    const uint32_t cw[4] = {__byte_perm(a01, a23, 0x5410), __byte_perm(a01, a23, 0x7632),
                            __byte_perm(b01, b23, 0x5410), __byte_perm(b01, b23, 0x7632)};
    // word br of local row kk sits at slot (br + kk / 8) % 16, so the lanes of
    // a warp (bc = 0..15, two br) spread over the banks
#pragma unroll
    for (int q = 0; q < 4; ++q) tc[8 * bc + 4 * g + q][(br + bc) & 15] = cw[q];
  }
  __syncthreads();
  // output rows k0 .. k0 + kKmajK - 1, 64 bytes (rows r0 .. r0 + 63) each per
  // plane: four threads per row, each decoding and storing 16 rows' bytes, so a
  // warp stores 8 rows x 64 bytes per plane.  The tile's 64 rows lie in one
  // 512-column block (b, width w).
  const int c = t & 3, r = r0 + 16 * c;
  const int blk = r0 & ~511, wb = min(512, ldt - blk);
  const uint32_t lane4 = (uint32_t)(t & 31) << 2;
  uint32_t la4[4], L4[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    la4[j] = ((const uint32_t *)s_la4)[4 * c + j];
    L4[j] = ((const uint32_t *)s_L4)[4 * c + j];
  }
#pragma unroll
  for (int pass = 0; pass < kKmajK / 64; ++pass) {
    const int kk = pass * 64 + (t >> 2), k = k0 + kk, rot = kk >> 3;
    if (k < K && r < ldt) {
      uint32_t vm[4], ve[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // rows 16c + 4j .. + 3: byte i of lw is row i's lsb + 64 (0 for zero / NaR)
        uint32_t mw, lw;
        kmaj_decode4(tc[kk][(4 * c + j + rot) & 15], s_tab, lane4, mw, lw);
        // per byte, lw | 0x80 minus L4 (or la4) cannot borrow from the next byte
        // (lw | 0x80 >= 128 > L4, la4); its bit 7 is lw >= L4, which also leaves
        // out zero and NaR (lw = 0 < 1 <= L4), spread to the byte by the
        // permute's sign replication
        const uint32_t x = lw | 0x80808080u;
        const uint32_t keep = byte_signs(x - L4[j]);
        vm[j] = mw & keep;
        ve[j] = (x - la4[j]) & 0x7F7F7F7Fu & keep;   // lsb - la
      }
      uint8_t *o = dme + (size_t)k * 2 * ldt + 2 * blk + (r - blk);
      *(uint4 *)o = make_uint4(vm[0], vm[1], vm[2], vm[3]);
      *(uint4 *)(o + wb) = make_uint4(ve[0], ve[1], ve[2], ve[3]);
    }
  }
}

__global__ void __launch_bounds__(256, 4) k_kmajor_bp8(const uint8_t *__restrict__ src, int rows, int K,
                                                    uint8_t *__restrict__ dme, int ldt,
                                                    const int4 *__restrict__ st, const int *__restrict__ Lr,
                                                    int *__restrict__ hr64) {
  extern __shared__ __align__(16) uint32_t kms[];
  uint32_t(*tc)[17] = (uint32_t(*)[17])kms;                       // [k][row / 4] code words, one pad word
  uint8_t *s_tab = (uint8_t *)(kms + kKmajK * 17);                 // kKmajTable bytes (kmaj_decode4)
  __shared__ __align__(16) uint8_t s_la4[64], s_L4[64];           // per tile row: la + 64, L + 64
  const int t = threadIdx.x;
  {
    int m, e;
    posit_to_me<8, 2>((uint32_t)t, m, e);
    // bp8 lsb exponents lie in [-24, 24]: the entry of a nonzero code is nonzero
    const uint16_t d = m ? (uint16_t)(((e + 64) << 8) | (uint8_t)(int8_t)m) : (uint16_t)0;
    for (int l = 0; l < 32; ++l) *(uint16_t *)(s_tab + (t >> 1) * 128 + 4 * l + 2 * (t & 1)) = d;
  }
  const int br = t >> 4, bc = t & 15;   // rows r0 + 4br .. + 3, columns k0 + 8bc .. + 7
  const bool vec = (K & 7) == 0 && (((uintptr_t)src) & 7u) == 0;
  const int tk = (K + kKmajK - 1) / kKmajK, tr = (ldt + 63) / 64;
  const long long ntiles = (long long)tk * tr, g = gridDim.x;
  // three fetch buffers in rotation, the loop unrolled by three: each buffer is
  // refilled (tile + 3g) right after its tile is written, so two tiles' loads
  // are in flight while one is worked on, and no register waits on a load
  // before its tile comes up
  KmajFetch fa, fb, fc;
  long long tile = blockIdx.x;
  kmaj_fetch(tile, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fa);
  kmaj_fetch(tile + g, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fb);
  kmaj_fetch(tile + 2 * g, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fc);
  for (; tile < ntiles; tile += 3 * g) {
    kmaj_tile(tile, tk, rows, K, dme, ldt, st, hr64, t, br, bc, fa, tc, s_tab, s_la4, s_L4);
    kmaj_fetch(tile + 3 * g, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fa);
    if (tile + g >= ntiles) break;
    kmaj_tile(tile + g, tk, rows, K, dme, ldt, st, hr64, t, br, bc, fb, tc, s_tab, s_la4, s_L4);
    kmaj_fetch(tile + 4 * g, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fb);
    if (tile + 2 * g >= ntiles) break;
    kmaj_tile(tile + 2 * g, tk, rows, K, dme, ldt, st, hr64, t, br, bc, fc, tc, s_tab, s_la4, s_L4);
    kmaj_fetch(tile + 5 * g, ntiles, tk, src, rows, K, vec, st, Lr, t, br, bc, fc);
  }
}

// Tail corrections of the narrow form (bp8, unscaled), the same sums as
// k_tc_corr read from the other operand's decoded K-major copy:
//   C[s][y] = sum over tail elements (x, k) of row x (slot s):  v(X[x,k]) * v(Y[y,k])
// in units of 2^(la_x + la_y).  Side 0 (A's tail rows) reads all of B; side 1
// (B's tail rows) reads A's main part -- its copy has A's own tail elements
// zeroed -- so the two sides add up to A.B - A_main.B_main.
// One warp per slot, no block barrier.  The warp lists up to kCorrChunk of the
// slot's tail elements in its own shared memory (column k, m_a, lsb_a - la_x)
// and takes the columns in passes of kCorrPass: for each tail element, lane 0
// streams that pass's block of row k (its M bytes, then its E bytes: one
// bulk copy; two copies per element, one per plane, ran at half the rate
// beside the GEMM) into the warp's ring of kCorrRing shared-memory stages (one
// mbarrier per stage, kCorrRing elements in flight), and each lane adds the
// terms of its kCorrCols columns from the stage (the register-load form was bound by the
// latency of its loads).  A term is (m_a << ea) * (m << e) with ea = lsb_a -
// la_x <= emax (the slot's largest) and e = lsb - la_y (hr: the widest row
// range hb - la among the pass's columns, hb the largest binade, per 64 rows
// from the copy).  A factor m << e is v / 2^la_y with |v| < 2^(hb + 1), so
// |m << e| < 2^(hr + 1); and |m_a| < 2^4 (at most 3 fraction bits), so
// |m_a << ea| < 2^(emax + 4): |term| < 2^(emax + hr + 5), and a sum of T <
// 2^lgT terms stays inside int64 while emax + hr + lgT <= 58 (two's
// complement words).  Then one 32 x 32 -> 64-bit multiply-add per term when
// both factors fit int32 (emax <= 27, hr <= 30), else a 64-bit shift of m_a m.
// Otherwise 128-bit shifts.  Every wait is bounded: a timeout records code 32
// in g_tc_error, waits (bounded) for the warp's copies in flight and ends the
// warp.
constexpr int kCorrCols = 16, kCorrChunk = 256, kCorrPass = 32 * kCorrCols, kCorrRing = 4, kCorrWarps = 8;
static_assert(kCorrPass == 512, "k_kmajor_bp8 lays its copies out in blocks of 512 columns");
// Each warp's region: the ring's stages, the list, the barriers; rounded up to
// 16 bytes, so that every warp's stages stay 16-byte aligned for the bulk
// copies and the lanes' 16-byte loads (an odd ring otherwise shifts them by 8).
constexpr size_t kCorrWarpSmem =
    (2 * (size_t)kCorrRing * kCorrPass + (size_t)kCorrChunk * 8 + kCorrRing * 8 + 15) / 16 * 16;
static_assert(kCorrWarpSmem % 16 == 0 && (2 * (size_t)kCorrRing * kCorrPass) % 16 == 0, "16-byte stages");
constexpr size_t kCorrSmem = kCorrWarps * kCorrWarpSmem;

struct CorrT {
  const uint8_t *X;
  const uint8_t *Yme;   // the other operand's K-major copy, [K][2 ldt] (M and E per 512-column block)
  int Yrows, ldt;
  const int4 *xst;
  const int4 *seg;
  const int *tails;
  const TcCounters *ctr;
  const int *yhr;   // the other operand's widest row range hb - la per 64 rows
  int cap;
  ulonglong2 *Cout;
};

enum { kCorrMul = 0, kCorrShift = 1, kCorrWide = 2 };

// The warp's shared memory: the ring's M and E stages, the list, the barriers.
struct CorrWarp {
  uint8_t *rme;   // stage s: [2 kCorrPass] bytes at s * 2 kCorrPass (the pass's M bytes, then its E bytes)
  int2 *lst;
  uint64_t *bar;
  uint32_t g;   // bulk copies issued so far (stage g % kCorrRing, phase (g / kCorrRing) & 1)
};

// Lane 0: the copy of tail element `k`'s pass block (its `bytes` M bytes and
// `bytes` E bytes, contiguous) into stage g % kCorrRing.
__device__ __forceinline__ void corr_issue(const CorrT &c, CorrWarp &w, uint32_t g, int k, int y0, int bytes) {
  const int st = (int)(g % kCorrRing);
  mbar_expect_tx(&w.bar[st], 2u * (uint32_t)bytes);
  bulk_g2s(w.rme + st * 2 * kCorrPass, c.Yme + (size_t)k * 2 * c.ldt + 2 * (size_t)y0, 2u * (uint32_t)bytes,
           &w.bar[st]);
}

// One pass (columns y0 .. y0 + kCorrPass - 1) of one slot.  Returns false
// after a timed-out wait (the warp's copies in flight have been waited for).
template <int MODE>
__device__ __forceinline__ bool corr_pass(const CorrT &c, CorrWarp &w, int4 sg, int la_x, int K, int y0, int lane,
                                          ulonglong2 *__restrict__ o) {
  constexpr bool WIDE = MODE == kCorrWide;
  using Acc = typename std::conditional<WIDE, unsigned __int128, unsigned long long>::type;
  Acc acc[kCorrCols];
#pragma unroll
  for (int q = 0; q < kCorrCols; ++q) acc[q] = 0;
  const int T = sg.y;
  const int bytes = min(kCorrPass, c.ldt - y0);   // a multiple of 16
  const bool mine = 16 * lane < bytes;            // this lane's 16 columns lie in the slice
  for (int c0 = 0; c0 < T; c0 += kCorrChunk) {
    const int n = min(kCorrChunk, T - c0);
    if (T > kCorrChunk) {   // longer lists are re-read per chunk (no copy in flight here)
      __syncwarp();
      for (int t = lane; t < n; t += 32) {
        const int k = c.tails[sg.x + c0 + t];
        int m, e;
        posit_to_me<8, 2>((uint32_t)c.X[(size_t)sg.z * K + k], m, e);
        w.lst[t] = make_int2(k, (m & 0xFFFF) | ((e - la_x) << 16));
      }
      __syncwarp();
    }
    const uint32_t g0 = w.g;
    if (lane == 0)
      for (int j = 0; j < min(kCorrRing, n); ++j) corr_issue(c, w, g0 + j, w.lst[j].x, y0, bytes);
    for (int t = 0; t < n; ++t) {
      const uint32_t gi = g0 + t;
      const int st = (int)(gi % kCorrRing);
      if (!mbar_wait_warp(&w.bar[st], (gi / kCorrRing) & 1u, 32)) {
        // wait, bounded, for the copies still in flight, then give up
        if (lane == 0)
          for (int u = t; u < min(n, t + kCorrRing); ++u) {   // issued: 0 .. t + kCorrRing - 1
            const uint32_t gu = g0 + u;
            const long long t1 = clock64();
            while (!mbar_try_wait(&w.bar[gu % kCorrRing], (gu / kCorrRing) & 1u) && clock64() - t1 < DRAIN_LIMIT)
              __nanosleep(256);
          }
        __syncwarp();
        return false;
      }
      if (mine) {
        const uint4 wm = *(const uint4 *)(w.rme + st * 2 * kCorrPass + 16 * lane);
        const uint4 we = *(const uint4 *)(w.rme + st * 2 * kCorrPass + bytes + 16 * lane);
        const int me = w.lst[t].y;
        const int ma = (int)(short)(me & 0xFFFF), ea = me >> 16;
        const int a32 = (int)((unsigned)ma << (ea & 31));   // used when ea <= 27
#pragma unroll
        for (int q = 0; q < kCorrCols; ++q) {
          const uint32_t wmq = q < 4 ? wm.x : q < 8 ? wm.y : q < 12 ? wm.z : wm.w;
          const uint32_t weq = q < 4 ? we.x : q < 8 ? we.y : q < 12 ? we.z : we.w;
          const int m = (int)(int8_t)(wmq >> (8 * (q & 3)));
          const int e = (int)((weq >> (8 * (q & 3))) & 0xFFu);
          if (MODE == kCorrWide) acc[q] += (unsigned __int128)(__int128)(ma * m) << min(ea + e, 127);
          else if (MODE == kCorrShift) acc[q] += (unsigned long long)(long long)(ma * m) << (ea + e);
          else acc[q] += (unsigned long long)((long long)a32 * (long long)(int)((unsigned)m << e));
        }
      }
      __syncwarp();   // every lane is done with stage st
      if (lane == 0 && t + kCorrRing < n) corr_issue(c, w, gi + kCorrRing, w.lst[t + kCorrRing].x, y0, bytes);
    }
    w.g = g0 + (uint32_t)n;
  }
  const int y = y0 + kCorrCols * lane;
  if (y < c.Yrows) {
#pragma unroll
    for (int q = 0; q < kCorrCols; ++q) {
      if (y + q >= c.Yrows) continue;
      if (WIDE) o[q] = make_ulonglong2((unsigned long long)acc[q], (unsigned long long)((unsigned __int128)acc[q] >> 64));
      else o[q] = make_ulonglong2((unsigned long long)acc[q], (unsigned long long)((long long)acc[q] >> 63));
    }
  }
  return true;
}

// The 128-bit form out of line (rare: rows spanning more than ~50 binades).
__device__ __noinline__ bool corr_pass_wide(const CorrT &c, CorrWarp &w, int4 sg, int la_x, int K, int y0, int lane,
                                            ulonglong2 *__restrict__ o) {
  return corr_pass<kCorrWide>(c, w, sg, la_x, K, y0, lane, o);
}

__global__ void __launch_bounds__(32 * kCorrWarps, 2) k_tc_corr_t(const CorrT s0, const CorrT s1, int K) {
  extern __shared__ __align__(16) uint8_t kcs[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *base = kcs + warp * kCorrWarpSmem;
  CorrWarp w;
  w.rme = base;
  w.lst = (int2 *)(base + 2 * kCorrRing * kCorrPass);
  w.bar = (uint64_t *)(base + 2 * kCorrRing * kCorrPass + kCorrChunk * 8);
  w.g = 0;
  if (lane == 0) {
    for (int r = 0; r < kCorrRing; ++r) mbar_init(&w.bar[r], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  // Work units: (slot, 512-column pass), slot-major, taken one at a time from
  // a counter (TcCounters v[8] of side 0, zeroed with the counters): slots hold
  // 2 to ~80 tail elements, and a fixed split left most warps idle behind a few.
  const int n0 = min(s0.ctr->v[0], s0.cap), n1 = min(s1.ctr->v[0], s1.cap);
  const int np0 = (s0.Yrows + kCorrPass - 1) / kCorrPass, np1 = (s1.Yrows + kCorrPass - 1) / kCorrPass;
  const long long nu0 = (long long)n0 * np0, nu = nu0 + (long long)n1 * np1;
  int *queue = const_cast<int *>(&s0.ctr->v[8]);
  int cur = -1;   // the slot item whose list is loaded
  int4 sg = make_int4(0, 0, 0, 0);
  int la_x = 0, em = 0, lgT = 0;
  for (;;) {
    long long u = 0;
    if (lane == 0) u = atomicAdd(queue, 1);
    u = __shfl_sync(0xFFFFFFFFu, u, 0);
    if (u >= nu) break;
    const bool second = u >= nu0;
    const CorrT &c = second ? s1 : s0;
    const long long uu = second ? u - nu0 : u;
    const int np = second ? np1 : np0;
    const int sl = (int)(uu / np), y0 = (int)(uu % np) * kCorrPass;
    const int item = second ? n0 + sl : sl;
    if (item != cur) {
      cur = item;
      sg = c.seg[sl];
      const int x = sg.z, T = sg.y;
      la_x = c.xst[x].x;
      // the first chunk of the list, and the slot's largest tail exponent
      em = 0;
      __syncwarp();
      for (int t = lane; t < min(T, kCorrChunk); t += 32) {
        const int k = c.tails[sg.x + t];
        int m, e;
        posit_to_me<8, 2>((uint32_t)c.X[(size_t)x * K + k], m, e);
        w.lst[t] = make_int2(k, (m & 0xFFFF) | ((e - la_x) << 16));   // e >= la_x: the row's min lsb
        em = max(em, e - la_x);
      }
      for (int t = kCorrChunk + lane; t < T; t += 32) {
        int m, e;
        posit_to_me<8, 2>((uint32_t)c.X[(size_t)x * K + c.tails[sg.x + t]], m, e);
        em = max(em, e - la_x);
      }
      em = __reduce_max_sync(0xFFFFFFFFu, em);
      __syncwarp();
      lgT = 32 - __clz(max(T, 1));   // >= ceil(log2(T + 1))
    }
    // the widest row range among this pass's 512 columns (8 blocks of 64)
    int hr = lane < kCorrPass / 64 && y0 + 64 * lane < c.Yrows ? c.yhr[y0 / 64 + lane] : 0;
    hr = __reduce_max_sync(0xFFFFFFFFu, hr);
    const int mode = em + hr + lgT > 58 ? kCorrWide : (em <= 27 && hr <= 30) ? kCorrMul : kCorrShift;
    ulonglong2 *o = c.Cout + (size_t)sl * c.Yrows + y0 + kCorrCols * lane;
    bool ok;
    if (mode == kCorrMul) ok = corr_pass<kCorrMul>(c, w, sg, la_x, K, y0, lane, o);
    else if (mode == kCorrShift) ok = corr_pass<kCorrShift>(c, w, sg, la_x, K, y0, lane, o);
    else ok = corr_pass_wide(c, w, sg, la_x, K, y0, lane, o);
    if (!ok) return;
    if (sg.y > kCorrChunk) cur = -1;   // the list buffer now holds a later chunk
  }
}

// ----------------------------------------------------------------- fixup ---
template <int FMT>
__global__ void __launch_bounds__(256) k_tc_fixup(GemmArgs a, const int4 *__restrict__ sta,
                                                  const int4 *__restrict__ stb, const int *__restrict__ slotA,
                                                  const int *__restrict__ slotB, const TcCounters *__restrict__ cA,
                                                  const TcCounters *__restrict__ cB) {
  // Every output is 0 when an operand has no nonzero row; and when the
  // global bounds already make every pair exact there is nothing to redo.
  if (!cA->v[5] || !cB->v[5]) return;
  if (*(volatile int *)&g_tc_error != 0) return;   // k_tc_finish wrote NaR everywhere
  const int min_la = (BIG - cA->v[2]) + (BIG - cB->v[2]);
  const int max_w = cA->v[3] + cB->v[3] + 2 + ceil_log2_int(a.K) + 1;
  if (min_la + 96 >= 0 && max_w <= 127 && !cA->v[4] && !cB->v[4]) return;
  size_t n = (size_t)a.M * a.N;
  for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < n; o += (size_t)gridDim.x * blockDim.x) {
    int i = (int)(o / a.N), j = (int)(o % a.N);
    int4 ra = sta[i], rb = stb[j];
    if (!(ra.z && rb.z)) continue;
    if (tc_exact(ra, rb, slotA[i], slotB[j], a.K)) continue;
    uint32_t code;
    slow_output<FMT>(a, i, j, &code, a.quire ? a.quire + ((size_t)i * a.N + j) * a.nlimbs : nullptr);
    store_output(a, i, j, code);
    for (int e = 0; e < a.n_extra; ++e) a.extra_out[e][(size_t)i * a.ldo + a.extra_col0 + j] = code;
  }
  if (a.n_extra) __threadfence_system();
}

// ------------------------------------------------------------ host side ---
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// [S][rows][Kp] int8 planes; box {BK (K), box_rows, S}; 64-byte swizzle.
int make_plane_map(CUtensorMap *m, void *base, int Kp, int rows, int S, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(kECuda, "quire_gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)S};
  cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)Kp * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)S};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  BK == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kECuda, "quire_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return kOk;
}

inline size_t al(size_t v) { return (v + 255) / 256 * 256; }

struct TcLayout {
  int S, Kp, nkb, capA, capB, pool, ldtA, ldtB;
  size_t planesA, planesB, LA, LB, slotA, slotB, segA, segB, tailA, tailB, ctr, CA, CB, TA, TB, HA, HB, part, total;
};

// K at and above which unscaled bp8 takes the narrow form on its own (algo 0,
// 2, 3): 4 digit-pair MMAs instead of 9 per K block, against tail lists of a
// few tens of elements per row for rows whose values spread like N(0, 1)
// (15-bit window) corrected beside the GEMM.
constexpr int kNarrowMinK = 16384;

// Digit planes of a call: 2 (narrow bp8 form), 3 (wide bp8) or 4 (bp16).
// algo 4 forces the narrow form and algo 5 the wide one (bp8).
int tc_planes(int fmt, int K, bool scaled, int algo) {
  if (fmt != 8) return 4;
  if (algo == 4) return 2;
  if (algo == 5) return 3;
  return (!scaled && K >= kNarrowMinK) ? 2 : 3;
}

// Correction buffers hold at most this many bytes per side; tail rows beyond
// the cap are finished by the fixup kernel instead.
constexpr size_t kCorrBudget = size_t(512) << 20;

// Which tiles run whole and which are split along K.  Tiles are indexed in
// tile_coords order; tiles [0, whole) run whole, tiles [whole, ntiles) in `split`
// chunks of kbc K blocks each, their int64 partial sums added by k_tc_finish.
//  * K longer than one exact int32 chunk: every tile is split (the minimum).
//  * otherwise the full waves run whole and only the last, partial wave is
//    split -- as many ways as fit in one wave -- so the machine stays full to
//    the end instead of idling through a mostly empty last wave.
struct TcSchedule {
  int MM, BN, QW, ntn, ntiles, whole, split, kbc;
};

int tc_wave_capacity(bool pair);

TcSchedule tc_schedule(int S, int M, int N, int nkb, bool pair) {
  TcSchedule sc{};
  sc.MM = pair ? 2 * BM : BM;
  sc.BN = S == 2 ? Cfg<2>::BN : (S == 3 ? Cfg<3>::BN : Cfg<4>::BN);
  sc.QW = S == 2 ? Cfg<2>::QW : (S == 3 ? Cfg<3>::QW : Cfg<4>::QW);
  sc.ntn = (N + sc.BN - 1) / sc.BN;
  sc.ntiles = sc.ntn * ((M + sc.MM - 1) / sc.MM);
  const int exact = (S == 2 ? Cfg<2>::KCHUNK : (S == 3 ? Cfg<3>::KCHUNK : Cfg<4>::KCHUNK)) / BK;
  const int min_split = (nkb + exact - 1) / exact;
  const int P = std::max(1, tc_wave_capacity(pair));
  if (min_split > 1) {
    sc.whole = 0;
    sc.split = min_split;
  } else {
    const int R = sc.ntiles % P;
    int sp = R ? P / R : 1;
    sp = std::min(sp, std::max(1, nkb / 16));   // keep at least 16 K blocks per chunk
    sc.split = sp;
    sc.whole = sp > 1 ? sc.ntiles - R : sc.ntiles;
  }
  sc.kbc = (nkb + sc.split - 1) / sc.split;
  sc.split = (nkb + sc.kbc - 1) / sc.kbc;   // every chunk non-empty
  if (sc.split == 1) sc.whole = sc.ntiles;
  return sc;
}

// Exact main sums of one GEMM: QW int64 words per output of the whole tiles,
// then per output and K chunk of the split tiles.
size_t tc_qbuf_bytes(const TcSchedule &sc) {
  return 8 * (size_t)sc.QW * ((size_t)sc.whole + (size_t)(sc.ntiles - sc.whole) * sc.split) * sc.MM * sc.BN;
}

// Workspace layout for a call with S digit planes.  The narrow form (S = 2)
// adds the K-major copies of both operands' codes and a deeper tail pool.
TcLayout tc_layout(int fmt, int M, int N, int K, int S) {
  TcLayout L{};
  L.S = S;
  L.Kp = (K + 127) / 128 * 128;
  L.nkb = L.Kp / BK;
  L.capA = (int)std::min<size_t>((size_t)M, std::max<size_t>(1, kCorrBudget / (16 * (size_t)std::max(N, 1))));
  L.capB = (int)std::min<size_t>((size_t)N, std::max<size_t>(1, kCorrBudget / (16 * (size_t)std::max(M, 1))));
  L.pool = std::max(65536, (S == 2 ? 128 : 8) * std::max(M, N));
  L.ldtA = (M + 15) / 16 * 16;
  L.ldtB = (N + 15) / 16 * 16;
  size_t o = 0;
  L.planesA = o; o += al((size_t)L.S * M * L.Kp);
  L.planesB = o; o += al((size_t)L.S * N * L.Kp);
  L.LA = o; o += al(4 * (size_t)M);
  L.LB = o; o += al(4 * (size_t)N);
  L.slotA = o; o += al(4 * (size_t)M);
  L.slotB = o; o += al(4 * (size_t)N);
  L.segA = o; o += al(16 * (size_t)L.capA);
  L.segB = o; o += al(16 * (size_t)L.capB);
  L.tailA = o; o += al(4 * (size_t)L.pool);
  L.tailB = o; o += al(4 * (size_t)L.pool);
  L.ctr = o; o += 256;
  L.CA = o; o += al(16 * (size_t)L.capA * N);
  L.CB = o; o += al(16 * (size_t)L.capB * M);
  L.TA = L.TB = L.HA = L.HB = 0;
  if (S == 2) {   // two byte planes (mantissa, relative lsb) per copy; row ranges per 64 rows
    L.TA = o; o += al(2 * (size_t)K * L.ldtA);
    L.TB = o; o += al(2 * (size_t)K * L.ldtB);
    L.HA = o; o += al(4 * (size_t)(L.ldtA / 16 + 4));
    L.HB = o; o += al(4 * (size_t)(L.ldtB / 16 + 4));
  }
  // room for either pairing's main sums (chosen at launch)
  L.part = o;
  o += al(std::max(tc_qbuf_bytes(tc_schedule(L.S, M, N, L.nkb, false)),
                   tc_qbuf_bytes(tc_schedule(L.S, M, N, L.nkb, M > BM && BK == 64))));
  L.total = o;
  return L;
}

template <int S, bool PAIR>
cudaError_t tc_kernel_attr() {   // once per device
  static std::atomic<bool> done[128];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 0 && dev < 128 && done[dev].load()) return cudaSuccess;
  err = cudaFuncSetAttribute(k_quire_gemm_tc<S, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<S, PAIR>::SMEM);
  // the whole unified L1 as shared memory: with the smallest carveout that
  // holds the CTA, the narrow form's copy and correction blocks found no
  // room beside it
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(k_quire_gemm_tc<S, PAIR>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
  if (err == cudaSuccess && dev >= 0 && dev < 128) done[dev].store(true);
  return err;
}

cudaLaunchConfig_t pair_config(dim3 grid, cudaStream_t s, size_t smem, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Tiles (CTAs, or CTA pairs) resident at once: the SM count, or the number of
// co-resident 2-CTA clusters of the paired kernel on this device (cached).
int tc_wave_capacity(bool pair) {
  const int sms = sm_count();
  if (!pair) return sms;
  static std::atomic<int> cache[128];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return sms / 2;
  int v = cache[dev].load();
  if (v > 0) return v;
  int n = 0;
  if (tc_kernel_attr<3, true>() == cudaSuccess) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pair_config(dim3(2 * 1024, 1, 1), nullptr, Cfg<3, true>::SMEM, attr);
    if (cudaOccupancyMaxActiveClusters(&n, k_quire_gemm_tc<3, true>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  v = n > 0 ? n : sms / 2;
  cache[dev].store(v);
  return v;
}

// One launch over `ntiles` linear tiles starting at p.tile0, p.split K chunks each.
template <int S, bool PAIR>
int launch_tc_gemm_kernel(const CUtensorMap &ma, const CUtensorMap &mb, const TcParams &p, int ntiles,
                          cudaStream_t s) {
  using C = Cfg<S, PAIR>;
  cudaError_t attr_err = tc_kernel_attr<S, PAIR>();
  if (attr_err != cudaSuccess)
    return set_error(kECuda, "quire_gemm: cannot set shared memory size: %s", cudaGetErrorString(attr_err));
  // persistent: at most one resident CTA (pair) per SM (pair), each striding
  // over the launch's (tile, K chunk) units
  const long long units = (long long)ntiles * p.split;
  if (units > 0x7FFFFFFFLL) return set_error(kERange, "quire_gemm: too many K chunks");
  const int ncta = (int)std::min<long long>(units, std::max(1, tc_wave_capacity(PAIR)));
  dim3 grid((unsigned)((PAIR ? 2 : 1) * ncta), 1, 1);
  if (!PAIR) {
    k_quire_gemm_tc<S, false><<<grid, THREADS, C::SMEM, s>>>(ma, mb, p);
    return check_launch("quire_gemm_tc");
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pair_config(grid, s, C::SMEM, attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_quire_gemm_tc<S, true>, ma, mb, p);
  if (e != cudaSuccess) return set_error(kECuda, "quire_gemm_tc (paired): %s", cudaGetErrorString(e));
  return check_launch("quire_gemm_tc");
}

// Launch shape of k_tc_finish for `ntiles` tiles and at most `cap` blocks:
// each tile cut into `parts` items (a power of two up to MM / 8 rows) until
// there are at least eight items per block.
template <int MM>
void finish_shape(int ntiles, int cap, int &grid, int &parts) {
  parts = 1;
  while (parts < MM / 8 && (long long)ntiles * parts < 8LL * cap) parts *= 2;
  grid = (int)std::max<long long>(1, std::min<long long>((long long)ntiles * parts, cap));
}

// A per-thread, per-device side stream (lowest priority) and events for the
// finish kernels that overlap the next GEMM launch.  Per thread, so a stream
// captured into a CUDA graph by one thread never shares it with another.
// Never destroyed: they live as long as the thread's CUDA context.
struct SideStream {
  cudaStream_t st = nullptr;
  cudaEvent_t ev[5] = {};   // 0, 1: finish forks; 2: join; 3: tail-correction fork; 4: corrections done
};

SideStream *side_stream() {
  constexpr int kDev = 64;
  thread_local SideStream ss[kDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDev) {
    cudaGetLastError();
    return nullptr;
  }
  SideStream &x = ss[dev];
  if (!x.st) {
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    cudaStream_t st = nullptr;
    if (cudaStreamCreateWithPriority(&st, cudaStreamNonBlocking, lo) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    for (cudaEvent_t &e : x.ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
      }
    x.st = st;
  }
  return &x;
}

// The GEMM in segments of tiles: all whole tiles but the last full wave, the
// last full wave, then the K-split remainder.  A segment's finish kernel runs
// on the side stream while the next segment's GEMM runs (its grid capped at
// two blocks per SM, so the GEMM's CTA still fits beside them) when that GEMM
// hides it: measured on B200, a tile's finish at two blocks per SM costs
// about half of one 64-deep K block of a full wave of tiles, so the rule is
// tiles <= 2 x the next segment's K blocks per tile (long K only: the
// 4096 x 4096 x 65536 GEMM overlaps, K <= 4864 does not).  Otherwise, and for
// the last segment, the finish runs on the caller's stream, which finally
// waits for the side stream.
template <int S, bool PAIR>
int launch_tc_schedule(const CUtensorMap &ma, const CUtensorMap &mb, TcParams p, const TcSchedule &sc,
                       int grid_finish, cudaStream_t s, cudaEvent_t corr_done,
                       const std::function<int(bool)> *after_first = nullptr) {
  using C = Cfg<S, PAIR>;
  struct Seg {
    int tile0, n, split, kbc;
  } seg[3];
  int nseg = 0;
  const int P = std::max(1, tc_wave_capacity(PAIR));
  SideStream *side = side_stream();
  if (sc.whole > 0) {
    if (side && sc.whole >= 2 * P && sc.whole - P <= 2 * p.nkb) {
      seg[nseg++] = {0, sc.whole - P, 1, p.nkb};
      seg[nseg++] = {sc.whole - P, P, 1, p.nkb};
    } else {
      seg[nseg++] = {0, sc.whole, 1, p.nkb};
    }
  }
  if (sc.whole < sc.ntiles) seg[nseg++] = {sc.whole, sc.ntiles - sc.whole, sc.split, sc.kbc};
  long long *qbuf = p.qbuf;
  p.ntn = sc.ntn;
  // corrections computed on the side stream: finishes there follow them in
  // stream order, the caller's stream waits for them before its first finish
  bool forked = corr_done != nullptr, corr_waited = false;
  int rc = kOk;
  for (int k = 0; k < nseg && rc == kOk; ++k) {
    p.tile0 = seg[k].tile0;
    p.split = seg[k].split;
    p.kb_per_chunk = seg[k].kbc;
    // every tile before this segment ran whole
    p.qbuf = qbuf + (size_t)seg[k].tile0 * C::QW * C::MM * C::BN;
    p.ntl = seg[k].n;
    rc = launch_tc_gemm_kernel<S, PAIR>(ma, mb, p, seg[k].n, s);
    if (rc) break;
    // work that runs beside the GEMM (it records corr_done): after the first
    // segment's CTAs, so that they are placed first
    // (told whether this is the only segment: then no later GEMM launch can be
    // held back by its blocks that wait for the GEMM's SMs)
    if (k == 0 && after_first && (rc = (*after_first)(nseg == 1)) != kOk) break;
    const bool on_s = k == nseg - 1 || !side || seg[k].n > 2 * seg[k + 1].kbc;
    cudaStream_t fs = on_s ? s : side->st;
    if (!on_s) {
      if (cudaEventRecord(side->ev[k], s) != cudaSuccess || cudaStreamWaitEvent(side->st, side->ev[k], 0) != cudaSuccess) {
        rc = set_error(kECuda, "quire_gemm: side stream: %s", cudaGetErrorString(cudaGetLastError()));
        break;
      }
      forked = true;
    }
    if (on_s && corr_done && !corr_waited) {
      if (cudaStreamWaitEvent(s, corr_done, 0) != cudaSuccess) {
        rc = set_error(kECuda, "quire_gemm: side stream: %s", cudaGetErrorString(cudaGetLastError()));
        break;
      }
      corr_waited = true;
    }
    int g = 1, parts = 1;
    finish_shape<C::MM>(seg[k].n, on_s ? grid_finish : std::min(grid_finish, 2 * sm_count()), g, parts);
    const size_t ssm = finish_staged_smem<C::MM, C::BN, C::QW>();
    if (on_s && p.split == 1 && !p.quire) {
      // the SMs are free: stream the sums through shared memory
      if (p.out_f32) k_tc_finish_staged<C::MM, C::BN, C::QW, true><<<g, 256, ssm, fs>>>(p, seg[k].n, parts);
      else k_tc_finish_staged<C::MM, C::BN, C::QW, false><<<g, 256, ssm, fs>>>(p, seg[k].n, parts);
    } else {
      if (p.out_f32) k_tc_finish<C::MM, C::BN, C::QW, true><<<g, 256, 0, fs>>>(p, seg[k].n, parts);
      else k_tc_finish<C::MM, C::BN, C::QW, false><<<g, 256, 0, fs>>>(p, seg[k].n, parts);
    }
    rc = check_launch("tc_finish");
  }
  if (forked) {
    // join, also on the error path: the caller's stream never runs ahead of the side stream
    if (cudaEventRecord(side->ev[2], side->st) != cudaSuccess || cudaStreamWaitEvent(s, side->ev[2], 0) != cudaSuccess)
      if (rc == kOk) rc = set_error(kECuda, "quire_gemm: side stream join: %s", cudaGetErrorString(cudaGetLastError()));
  }
  return rc;
}

}  // namespace

bool gemm_tc_supported(int fmt, int M, int N, int K) {
  (void)fmt;
  return M > 0 && N > 0 && K > 0 && (size_t)K <= (size_t)1 << 30 && M <= 65535 * BM;
}

// Enough for every plane form the call may take (scaled operands never take
// the narrow form on their own, but their size is not known here).
size_t gemm_tc_workspace(int fmt, int M, int N, int K, int algo) {
  const int s_unscaled = tc_planes(fmt, K, false, algo), s_scaled = tc_planes(fmt, K, true, algo);
  return std::max(tc_layout(fmt, M, N, K, s_unscaled).total, tc_layout(fmt, M, N, K, s_scaled).total);
}

// sta / stb are outputs here: the prep kernels write the row statistics.
// One operand's preparation (statistics, digit planes, bases, tail lists,
// counters) can be done alone (a_mode 2 for A, 3 for B) and reused by later
// calls with the same operand, M, N, K and workspace that prepare only the
// other one (a_mode 1 reuses A, 4 reuses B).
int launch_gemm_tc(const GemmArgs &a, int4 *sta, int4 *stb, void *ws, size_t ws_bytes, int algo, int a_mode,
                   cudaStream_t s) {
  // a_mode 0: prepare A and B and multiply; 1: A already prepared (reuse);
  // 2: prepare A only; 3: prepare B only; 4: B already prepared (reuse)
  const bool reuse_a = a_mode == 1, a_only = a_mode == 2, b_only = a_mode == 3, reuse_b = a_mode == 4;
  const bool single_sm = algo == 3;
  const int S = tc_planes(a.fmt, a.K, a.sa != nullptr || a.sb != nullptr, algo);
  // K-major corrections: the narrow form on unscaled operands (group-scaled
  // ones, which take the narrow form only when algo 4 asks, keep k_tc_corr)
  const bool kmajor = S == 2 && a.sa == nullptr && a.sb == nullptr;
  TcLayout L = tc_layout(a.fmt, a.M, a.N, a.K, S);
  if (ws_bytes < L.total) return set_error(kEWorkspace, "quire_gemm: tensor-core workspace too small");
  char *w = (char *)ws;
  int8_t *planesA = (int8_t *)(w + L.planesA), *planesB = (int8_t *)(w + L.planesB);
  int *LA = (int *)(w + L.LA), *LB = (int *)(w + L.LB);
  int *slotA = (int *)(w + L.slotA), *slotB = (int *)(w + L.slotB);
  int4 *segA = (int4 *)(w + L.segA), *segB = (int4 *)(w + L.segB);
  int *tailA = (int *)(w + L.tailA), *tailB = (int *)(w + L.tailB);
  TcCounters *cA = (TcCounters *)(w + L.ctr);
  TcCounters *cB = cA + 1;
  ulonglong2 *CA = (ulonglong2 *)(w + L.CA), *CB = (ulonglong2 *)(w + L.CB);
  long long *qbuf = (long long *)(w + L.part);

  // zero the counters of the operands prepared by this call
  cudaError_t e = (reuse_a || b_only) ? cudaMemsetAsync(cB, 0, sizeof(TcCounters), s)
                  : cudaMemsetAsync(cA, 0, ((a_only || reuse_b) ? 1 : 2) * sizeof(TcCounters), s);
  if (e != cudaSuccess) return set_error(kECuda, "quire_gemm: memset: %s", cudaGetErrorString(e));
  const int sms = sm_count();
  // the operands this call prepares, in one launch (an operand with rows = 0 is skipped)
  PrepOp pa{a.A, a.M, a.sa, sta, planesA, LA, slotA, segA, tailA, L.capA, cA};
  PrepOp pb{a.B, a.N, a.sb, stb, planesB, LB, slotB, segB, tailB, L.capB, cB};
  if (reuse_a || b_only) pa.rows = 0;
  if (reuse_b || a_only) pb.rows = 0;
  int rc = kOk;
  if (pa.rows + pb.rows > 0) {
    // one block per row at a time, sized to the row: a short row (the model
    // linears' K = 896) leaves most of a 256-thread block idle in both passes,
    // so short rows take 64 or 128 threads and more rows run at once; every
    // block is resident (1280 threads per SM at 48 registers)
    const int thr = a.K <= 2048 ? 64 : (a.K <= 8192 ? 128 : 256);
    const int g = std::min(pa.rows + pb.rows, sms * (1280 / thr));
    if (a.fmt == 16)
      k_tc_prep<16, 4><<<g, thr, 0, s>>>(pa, pb, a.K, L.Kp, a.G, a.group, L.pool);
    else if (S == 2)
      k_tc_prep<8, 2><<<g, thr, 0, s>>>(pa, pb, a.K, L.Kp, a.G, a.group, L.pool);
    else
      k_tc_prep<8, 3><<<g, thr, 0, s>>>(pa, pb, a.K, L.Kp, a.G, a.group, L.pool);
    rc = check_launch("tc_prep");
  }
  // The narrow form's decoded K-major copies of the operands prepared here --
  // B's whole, A's main part (its tail elements zeroed, by LA) -- and its tail
  // corrections from them.  With long K they run on the side stream beside the
  // GEMM, launched right after its first (persistent) segment, whose CTAs then
  // hold every SM and leave room for two copy blocks or one correction block
  // (2 x 26 or 50 KB of shared memory beside the GEMM's 178 KB; every kernel
  // asks for the whole L1 as shared memory); otherwise they run on the
  // caller's stream ahead of the GEMM.
  if (!rc && kmajor) {   // the shared-memory opt-ins, once per device
    static std::atomic<bool> attr_set[128];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128 ||
        (!attr_set[dev].load() &&
         (cudaFuncSetAttribute(k_kmajor_bp8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kKmajSmem) != cudaSuccess ||
          cudaFuncSetAttribute(k_tc_corr_t, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCorrSmem) != cudaSuccess ||
          cudaFuncSetAttribute(k_kmajor_bp8, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared) != cudaSuccess ||
          cudaFuncSetAttribute(k_tc_corr_t, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared) != cudaSuccess)))
      rc = set_error(kECuda, "quire_gemm: k-major kernels' attributes: %s", cudaGetErrorString(cudaGetLastError()));
    else
      attr_set[dev].store(true);
  }
  // the copies of the operands prepared here, on `st`, at most `cap` blocks each
  auto launch_copies = [&](cudaStream_t st, long long cap) -> int {
    auto kmg = [&](int K, int ldt) {
      const long long tiles = (long long)((K + kKmajK - 1) / kKmajK) * ((ldt + 63) / 64);
      return (unsigned)std::max<long long>(1, std::min<long long>(tiles, cap));
    };
    if (pa.rows) {
      if (cudaMemsetAsync(w + L.HA, 0, 4 * (size_t)(L.ldtA / 16 + 4), st) != cudaSuccess)
        return set_error(kECuda, "quire_gemm: memset: %s", cudaGetErrorString(cudaGetLastError()));
      k_kmajor_bp8<<<kmg(a.K, L.ldtA), 256, kKmajSmem, st>>>((const uint8_t *)a.A, a.M, a.K, (uint8_t *)(w + L.TA),
                                                             L.ldtA, sta, LA, (int *)(w + L.HA));
      const int r = check_launch("tc_kmajor");
      if (r) return r;
    }
    if (pb.rows) {
      if (cudaMemsetAsync(w + L.HB, 0, 4 * (size_t)(L.ldtB / 16 + 4), st) != cudaSuccess)
        return set_error(kECuda, "quire_gemm: memset: %s", cudaGetErrorString(cudaGetLastError()));
      k_kmajor_bp8<<<kmg(a.K, L.ldtB), 256, kKmajSmem, st>>>((const uint8_t *)a.B, a.N, a.K, (uint8_t *)(w + L.TB),
                                                             L.ldtB, stb, nullptr, (int *)(w + L.HB));
      return check_launch("tc_kmajor");
    }
    return kOk;
  };
  // the corrections (one warp per slot and column pass), on `st`, `grid` blocks
  auto launch_corr_t = [&](cudaStream_t st, int grid) -> int {
    const CorrT ca{(const uint8_t *)a.A, (const uint8_t *)(w + L.TB), a.N, L.ldtB, sta, segA, tailA, cA,
                   (const int *)(w + L.HB), L.capA, CA};
    const CorrT cb{(const uint8_t *)a.B, (const uint8_t *)(w + L.TA), a.M, L.ldtA, stb, segB, tailB, cB,
                   (const int *)(w + L.HA), L.capB, CB};
    // the kernel's work counter (side A's v[8]; a call that reuses A's prepared
    // state did not zero A's counters)
    if (cudaMemsetAsync(&cA->v[8], 0, sizeof(int), st) != cudaSuccess)
      return set_error(kECuda, "quire_gemm: memset: %s", cudaGetErrorString(cudaGetLastError()));
    k_tc_corr_t<<<grid, 32 * kCorrWarps, kCorrSmem, st>>>(ca, cb, a.K);
    return check_launch("tc_corr");
  };
  SideStream *oside = (!rc && kmajor && L.nkb >= 256 && !a_only && !b_only) ? side_stream() : nullptr;
  if (!rc && kmajor && !oside) rc = launch_copies(s, 4LL * sms);
  if (rc || a_only || b_only) return rc;

  // Paired SMs whenever the tile has a second 128-row half to work on.
  const bool pair = !single_sm && BK == 64 && a.M > BM;
  const int bnb = S == 2   ? (pair ? Cfg<2, true>::BNB : Cfg<2>::BNB)
                  : S == 3 ? (pair ? Cfg<3, true>::BNB : Cfg<3>::BNB)
                           : (pair ? Cfg<4, true>::BNB : Cfg<4>::BNB);
  CUtensorMap ma, mb;
  rc = make_plane_map(&ma, planesA, L.Kp, a.M, S, BM);
  if (rc) return rc;
  rc = make_plane_map(&mb, planesB, L.Kp, a.N, S, bnb);
  if (rc) return rc;

  TcParams p{};
  p.M = a.M; p.N = a.N; p.K = a.K; p.Kp = L.Kp; p.nkb = L.nkb;
  p.sta = sta; p.stb = stb; p.LA = LA; p.LB = LB; p.slotA = slotA; p.slotB = slotB;
  p.CA = CA; p.CB = CB;
  p.out = a.out; p.ldo = a.ldo; p.quire = a.quire; p.nlimbs = a.nlimbs; p.qbuf = qbuf;
  p.out_f32 = a.out_f32; p.ldf = a.ldf; p.re = a.re; p.ce = a.ce; p.bias = a.bias;
  p.n_extra = a.n_extra; p.extra_col0 = a.extra_col0;
  for (int e = 0; e < a.n_extra; ++e) p.extra_out[e] = a.extra_out[e];
  const TcSchedule sc = tc_schedule(S, a.M, a.N, L.nkb, pair);
  if (tc_qbuf_bytes(sc) > L.total - L.part) return set_error(kEWorkspace, "quire_gemm: sum buffer too small");
  size_t outs = (size_t)a.M * a.N;
  // k_tc_fixup almost always exits at once (the global row bounds show nothing
  // to redo): a small grid keeps that exit cheap; when there is work, its
  // blocks stride over all outputs
  int g = (int)std::min<size_t>((outs + 255) / 256, (size_t)sms * 2);
  const int gf = sms * 4;   // k_tc_finish: four blocks per SM are resident

  // tail corrections (the kernels read the tail-row counts on the device).
  // Only the finish kernels read them: with long K (64-deep K blocks >= 256)
  // they run on the side stream, at most two blocks per SM beside the GEMM's
  // first segment, instead of ahead of it.
  // The narrow form's corrections run on the caller's stream, ahead of the
  // GEMM: beside it, on the low-priority side stream, they were held back
  // until the GEMM's last CTAs were dispatched and then kept its last wave
  // from starting (their blocks' registers).
  SideStream *side = (L.nkb >= 256 && !kmajor) ? side_stream() : nullptr;
  if (side && (cudaEventRecord(side->ev[3], s) != cudaSuccess ||
               cudaStreamWaitEvent(side->st, side->ev[3], 0) != cudaSuccess)) {
    cudaGetLastError();
    side = nullptr;   // corrections on the caller's stream instead
  }
  const cudaStream_t cs = side ? side->st : s;
  if (kmajor) {
    // ahead of the GEMM, two 8-warp blocks per SM; beside it, from the hook below
    if (!oside) rc = launch_corr_t(s, sms * 2);
  } else {
    const int cy = side ? 2 : 64;
    const CorrSide ca{a.A, a.B, a.N, a.sa, a.sb, sta, stb, nullptr, segA, tailA, cA, L.capA, CA,
                      std::min(L.capA, side ? sms : sms * 2), std::min((a.N + 255) / 256, cy)};
    const CorrSide cb{a.B, a.A, a.M, a.sb, a.sa, stb, sta, LA, segB, tailB, cB, L.capB, CB,
                      std::min(L.capB, side ? sms : sms * 2), std::min((a.M + 255) / 256, cy)};
    const dim3 gc((unsigned)std::max(ca.gx, cb.gx), (unsigned)std::max(ca.gy, cb.gy), 2u);
    if (a.fmt == 8) k_tc_corr<8><<<gc, 256, 0, cs>>>(ca, cb, a.K, a.G, a.group);
    else k_tc_corr<16><<<gc, 256, 0, cs>>>(ca, cb, a.K, a.G, a.group);
    rc = check_launch("tc_corr");
  }
  cudaEvent_t corr_done = nullptr;
  std::function<int(bool)> beside;   // the narrow form's side work, launched after the first GEMM segment
  if (!rc && oside) {
    // the side stream starts after the prep (this record precedes the GEMM's launch)
    if (cudaEventRecord(oside->ev[3], s) != cudaSuccess || cudaStreamWaitEvent(oside->st, oside->ev[3], 0) != cudaSuccess)
      return set_error(kECuda, "quire_gemm: side stream: %s", cudaGetErrorString(cudaGetLastError()));
    beside = [&](bool only_segment) -> int {
      int r = launch_copies(oside->st, 2LL * sms);
      // one block per SM fits beside the GEMM's CTA; when the GEMM is a single
      // segment, a second block per SM (the work queue is dynamic) takes up
      // the SMs its CTAs leave, as no later GEMM segment waits behind them
      if (!r) r = launch_corr_t(oside->st, only_segment ? 2 * sms : sms);
      if (cudaEventRecord(oside->ev[4], oside->st) != cudaSuccess && !r)
        r = set_error(kECuda, "quire_gemm: side stream event: %s", cudaGetErrorString(cudaGetLastError()));
      return r;
    };
    corr_done = oside->ev[4];
  }
  if (side) {
    // the caller's stream always joins the side stream, on the error path too
    if (cudaEventRecord(side->ev[4], side->st) == cudaSuccess) corr_done = side->ev[4];
    else cudaGetLastError();
    if (rc || !corr_done) {
      if (corr_done) cudaStreamWaitEvent(s, corr_done, 0);
      else cudaStreamSynchronize(side->st);
      return rc ? rc : set_error(kECuda, "quire_gemm: side stream event failed");
    }
  }
  if (rc) return rc;
  if (S == 2)
    rc = pair ? launch_tc_schedule<2, true>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr)
              : launch_tc_schedule<2, false>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr);
  else if (S == 3)
    rc = pair ? launch_tc_schedule<3, true>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr)
              : launch_tc_schedule<3, false>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr);
  else
    rc = pair ? launch_tc_schedule<4, true>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr)
              : launch_tc_schedule<4, false>(ma, mb, p, sc, gf, s, corr_done, beside ? &beside : nullptr);
  if (rc) return rc;
  if (a.fmt == 8) k_tc_fixup<8><<<g, 256, 0, s>>>(a, sta, stb, slotA, slotB, cA, cB);
  else k_tc_fixup<16><<<g, 256, 0, s>>>(a, sta, stb, slotA, slotB, cA, cB);
  return check_launch("tc_fixup");
}

int tc_device_error(int *out) {
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof v);
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof zero);
  if (e != cudaSuccess) return set_error(kECuda, "bp_device_error: %s", cudaGetErrorString(e));
  *out = v;
  return kOk;
}

}  // namespace bp
