// bp_gemm_tc.cu -- exact quire GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in TMEM, operands staged by TMA).
//
// Same result as the CUDA-core path (and as dot_at_precision /
// bposit_fast.matmul_quire + quire256_to_bposit32, reference/bposit_ref.py:1028-1035,
// reference/bposit_fast.py:102-176, reference/bposit_ref.py:703-722), computed by
// exponent-sliced integer MMAs:
//
//  1. Per row r of an operand (row stats: min lsb exponent la_r, max binade
//     hb_r) choose a main base L_r = max(la_r, hb_r - SPAN + 1).  Every element
//     with lsb >= L_r is an integer X = v / 2^L_r with |X| < 2^SPAN, recoded
//     into S signed 8-bit digits X = sum_s d_s 256^s (d_s in [-128, 127]) and
//     stored as S int8 planes [S][rows][Kp] (k_tc_prep).  bp8: S = 3,
//     SPAN = 21; bp16: S = 4, SPAN = 29.
//  2. Elements below L_r (the rare far tail of a row) are left out of the
//     planes and added back exactly by k_tc_corr on CUDA cores:
//     A_tail * B + A_main * B_tail, one 128-bit sum per touched output.
//  3. The GEMM (k_quire_gemm_tc) issues, per 128-deep K block, S*S*4 int8
//     MMAs (128 x BN x 32) and accumulates digit pair (s, t) into TMEM
//     accumulator d = s + t.  K is cut into chunks of at most 32768 so every
//     int32 diagonal sum is exact (|sum| <= K * 49152 < 2^31).
//  4. The epilogue reads the 2S-1 diagonals, forms
//     Q = sum_d acc_d * 256^d (exact, 128-bit), moves it to the output's lsb
//     base la_i + la_j, adds the tail correction and rounds once to bposit32
//     (or stores Q per chunk for k_tc_reduce when K needed several chunks).
//  5. Outputs whose exact window exceeds 128 bits or that need per-term
//     truncation (products below 2^-96) are recomputed by k_tc_fixup with the
//     512-bit quire of the CUDA-core slow path.
//
// Warp roles in the GEMM (128 threads, one CTA per SM, 512 TMEM columns):
// warp 0 lane 0 issues TMA loads, warp 1 lane 0 issues MMAs, all four warps
// run the epilogue (warp w reads TMEM lanes 32w..32w+31 = tile rows).  All
// mbarrier waits are bounded; a timeout sets an error word and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "bp_gemm_common.cuh"
#include "bp_internal.cuh"

namespace bp {

__device__ int g_tc_error;   // nonzero after a bounded wait gave up

namespace {

constexpr int BM = 128, BK = 128, STAGES = 2, THREADS = 128;
constexpr int KCHUNK = 32768;                 // K per exact int32 chunk
constexpr long long WAIT_LIMIT = 4000000000LL; // cycles (~2 s) before a wait gives up

template <int S>
struct Cfg {
  static constexpr int BN = S == 3 ? 96 : 64;
  static constexpr int D = 2 * S - 1;
  static constexpr int A_BYTES = S * BM * BK;
  static constexpr int B_BYTES = S * BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + BN * 32;
  static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
  static_assert(D * BN <= 512, "TMEM budget");
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N");
};

struct TcParams {
  int M, N, K, Kp, nkb, kb_per_chunk, nchunks;
  const int4 *sta, *stb;
  const int *LA, *LB, *slotA, *slotB;
  const ulonglong2 *CA, *CB;   // tail corrections [slot][other dim], 128-bit
  uint32_t *out;
  int64_t ldo;
  uint32_t *quire;
  int nlimbs;
  ulonglong2 *partial;         // [chunk][M][N] when nchunks > 1
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

// Bounded wait: false (and the error word set) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int code) {
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > WAIT_LIMIT) {
      atomicOr(&g_tc_error, code);
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

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile with 128-byte swizzle: rows of 128 bytes, 8-row atoms
// 1024 bytes apart (SBO), leading offset 16 bytes (unused by the swizzle),
// descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
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

// Final value of one output from its main-part sum Q (lsb base L_i + L_j).
__device__ __forceinline__ void finish_output(const TcParams &p, int i, int j, unsigned __int128 Q, int4 ra,
                                              int4 rb, int Li, int Lj, int slot_i, int slot_j) {
  uint32_t *ob = p.out + (size_t)i * p.ldo + j;
  uint32_t *oq = p.quire ? p.quire + ((size_t)i * p.N + j) * p.nlimbs : nullptr;
  if (!(ra.z && rb.z)) {
    *ob = 0u;
    if (oq)
      for (int t = 0; t < p.nlimbs; ++t) oq[t] = 0u;
    return;
  }
  if (!tc_exact(ra, rb, slot_i, slot_j, p.K)) return;
  int sh = (Li - ra.x) + (Lj - rb.x);
  unsigned __int128 tot = Q << sh;
  if (slot_i >= 0) tot += u128(p.CA[(size_t)slot_i * p.N + j]);
  if (slot_j >= 0) tot += u128(p.CB[(size_t)slot_j * p.M + i]);
  write_fast_output(tot, ra.x + rb.x + 96, ob, oq, p.nlimbs);
}

// ----------------------------------------------------------------- GEMM ---
template <int S>
__global__ void __launch_bounds__(THREADS, 1)
    k_quire_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    TcParams p) {
  using C = Cfg<S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + STAGES * C::STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint32_t *tmem_slot = (uint32_t *)(tfull + 1);
  int4 *sstat = (int4 *)(smem + STAGES * C::STAGE_BYTES + 256);          // [BN] B-row stats
  int2 *sLs = (int2 *)(sstat + C::BN);                                    // [BN] {L, slot}

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * C::BN, m0 = blockIdx.y * BM, chunk = blockIdx.z;
  const int kb0 = chunk * p.kb_per_chunk;
  const int kb1 = min(p.nkb, kb0 + p.kb_per_chunk);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int c = threadIdx.x; c < C::BN; c += THREADS) {
    int j = n0 + c;
    sstat[c] = j < p.N ? p.stb[j] : make_int4(0, 0, 0, 0);
    sLs[c] = j < p.N ? make_int2(p.LB[j], p.slotB[j]) : make_int2(0, -1);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      for (int it = 0; it < nkb && ok; ++it) {
        int st = it % STAGES;
        uint32_t round = (uint32_t)(it / STAGES);
        ok = mbar_wait(&empty[st], (round & 1u) ^ 1u, 1);
        if (!ok) break;
        uint8_t *sa = smem + st * C::STAGE_BYTES;
        mbar_expect_tx(&full[st], C::STAGE_BYTES);
        tma_load_3d(sa, &tmA, &full[st], (kb0 + it) * BK, m0, 0);
        tma_load_3d(sa + C::A_BYTES, &tmB, &full[st], (kb0 + it) * BK, n0, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t init = 0u;
      for (int it = 0; it < nkb && ok; ++it) {
        int st = it % STAGES;
        uint32_t round = (uint32_t)(it / STAGES);
        ok = mbar_wait(&full[st], round & 1u, 2);
        if (!ok) break;
        tc_fence_after();
        uint32_t a0 = smem_u32(smem + st * C::STAGE_BYTES);
        uint32_t b0 = a0 + C::A_BYTES;
#pragma unroll
        for (int ks = 0; ks < BK / 32; ++ks) {
#pragma unroll
          for (int s = 0; s < S; ++s) {
            uint64_t ad = sw128_desc(a0 + s * BM * BK + ks * 32);
#pragma unroll
            for (int t = 0; t < S; ++t) {
              const int d = s + t;
              uint64_t bd = sw128_desc(b0 + t * C::BN * BK + ks * 32);
              umma_i8(tmem + d * C::BN, ad, bd, C::IDESC, (init >> d) & 1u);
              init |= 1u << d;
            }
          }
        }
        umma_commit(&empty[st]);
      }
      umma_commit(tfull);
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- epilogue
  ok = mbar_wait(tfull, 0, 4) && ok;
  tc_fence_after();
  const int r = warp * 32 + lane;
  const int i = m0 + r;
  int4 ra = make_int4(0, 0, 0, 0);
  int Li = 0, slot_i = -1;
  if (i < p.M) {
    ra = p.sta[i];
    Li = p.LA[i];
    slot_i = p.slotA[i];
  }
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
  for (int c0 = 0; c0 < C::BN; c0 += 16) {
    uint32_t v[C::D][16];
#pragma unroll
    for (int d = 0; d < C::D; ++d) tmem_ld16(trow + d * C::BN + c0, v[d]);
    tmem_ld_wait();
    if (!ok || i >= p.M) continue;
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int j = n0 + c0 + jj;
      if (j >= p.N) continue;
      unsigned __int128 Q = 0;
#pragma unroll
      for (int d = 0; d < C::D; ++d)
        Q += (unsigned __int128)(__int128)(long long)(int)v[d][jj] << (8 * d);
      if (p.nchunks > 1) {
        p.partial[((size_t)chunk * p.M + i) * p.N + j] = make_ulonglong2((unsigned long long)Q,
                                                                          (unsigned long long)(Q >> 64));
      } else {
        int2 ls = sLs[c0 + jj];
        finish_output(p, i, j, Q, ra, sstat[c0 + jj], Li, ls.x, slot_i, ls.y);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ----------------------------------------------------------- split-K sum ---
__global__ void __launch_bounds__(256) k_tc_reduce(TcParams p) {
  size_t n = (size_t)p.M * p.N;
  for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < n; o += (size_t)gridDim.x * blockDim.x) {
    int i = (int)(o / p.N), j = (int)(o % p.N);
    unsigned __int128 Q = 0;
    for (int c = 0; c < p.nchunks; ++c) Q += u128(p.partial[(size_t)c * n + o]);
    finish_output(p, i, j, Q, p.sta[i], p.stb[j], p.LA[i], p.LB[j], p.slotA[i], p.slotB[j]);
  }
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

// One warp per row: main base L, S digit planes (4 bytes per lane per plane
// per step), tail count, and a correction slot for rows with a tail.
template <int FMT, int S>
__global__ void __launch_bounds__(256) k_tc_prep(const void *__restrict__ codes, int rows, int K, int Kp,
                                                 const int32_t *__restrict__ sc, int G, int group,
                                                 const int4 *__restrict__ stats, int8_t *__restrict__ planes,
                                                 int *__restrict__ Lr, int *__restrict__ slot,
                                                 int *__restrict__ slot_row, int *__restrict__ counter, int cap) {
  constexpr int SPAN = 8 * S - 3;
  const int lane = threadIdx.x & 31;
  const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const size_t plane = (size_t)rows * Kp;
  for (long long r = warp; r < rows; r += nw) {
    int4 st = stats[r];
    int L = st.z ? max(st.x, st.y - (SPAN - 1)) : 0;
    int ntail = 0;
    int8_t *row = planes + (size_t)r * Kp;
    for (int k0 = lane * 4; k0 < Kp; k0 += 128) {
      uint32_t w[S];
#pragma unroll
      for (int s = 0; s < S; ++s) w[s] = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        int k = k0 + q;
        if (k >= K) break;
        ElemME x = decode_scaled<FMT>(load_code<FMT>(codes, (size_t)r * K + k), sc, (int)r, k, G, group);
        if (!x.m) continue;
        if (x.e < L) {
          ++ntail;
          continue;
        }
        int t = x.m * (1 << (x.e - L));
#pragma unroll
        for (int s = 0; s < S; ++s) {
          int d = (int)(int8_t)(uint8_t)(t & 0xFF);
          w[s] |= ((uint32_t)(uint8_t)d) << (8 * q);
          t = (t - d) >> 8;
        }
      }
#pragma unroll
      for (int s = 0; s < S; ++s) *(uint32_t *)(row + s * plane + k0) = w[s];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ntail += __shfl_xor_sync(0xFFFFFFFFu, ntail, o);
    if (lane == 0) {
      int sl = -1;
      if (ntail) {
        sl = atomicAdd(counter, 1);
        if (sl < cap) slot_row[sl] = (int)r;
        else sl = -2;
      }
      Lr[r] = L;
      slot[r] = sl;
    }
  }
}

// ------------------------------------------------------- tail correction ---
// For each tail row x of operand X (slot s), over all rows y of operand Y:
//   C[s][y] = sum over tail elements (x, k) of X:  v(X[x,k]) * v(Y[y,k])
// exactly, in units of 2^(la_x + la_y).  When YL is given, Y's own tail
// elements (lsb below YL[y]) are skipped (they were counted from Y's side).
template <int FMT>
__global__ void __launch_bounds__(256) k_tc_corr(const void *__restrict__ X, const void *__restrict__ Y, int Yrows,
                                                 int K, const int32_t *__restrict__ xs, const int32_t *__restrict__ ys,
                                                 int G, int group, const int4 *__restrict__ xst,
                                                 const int4 *__restrict__ yst, const int *__restrict__ XL,
                                                 const int *__restrict__ YL, const int *__restrict__ slot_row,
                                                 const int *__restrict__ counter, int cap,
                                                 ulonglong2 *__restrict__ Cout) {
  __shared__ int sk[256], sm[256], se[256];
  __shared__ int cnt;
  const int nslots = min(*counter, cap);
  for (int sl = blockIdx.x; sl < nslots; sl += gridDim.x) {
    const int x = slot_row[sl];
    const int4 sx = xst[x];
    const int Lx = XL[x];
    for (int y0 = blockIdx.y * 256; y0 < Yrows; y0 += gridDim.y * 256) {
      const int y = y0 + threadIdx.x;
      const bool valid = y < Yrows;
      const int4 sy = valid ? yst[y] : make_int4(0, 0, 0, 0);
      const int Ly = (YL && valid) ? YL[y] : -0x3FFFFFFF;
      unsigned __int128 acc = 0;
      for (int k0 = 0; k0 < K; k0 += 256) {
        if (threadIdx.x == 0) cnt = 0;
        __syncthreads();
        int k = k0 + threadIdx.x;
        if (k < K) {
          ElemME e = decode_scaled<FMT>(load_code<FMT>(X, (size_t)x * K + k), xs, x, k, G, group);
          if (e.m && e.e < Lx) {
            int pos = atomicAdd(&cnt, 1);
            sk[pos] = k;
            sm[pos] = e.m;
            se[pos] = e.e;
          }
        }
        __syncthreads();
        const int n = cnt;
        if (valid) {
          for (int t = 0; t < n; ++t) {
            const int kk = sk[t];
            ElemME f = decode_scaled<FMT>(load_code<FMT>(Y, (size_t)y * K + kk), ys, y, kk, G, group);
            if (!f.m || f.e < Ly) continue;
            long long P = (long long)sm[t] * f.m;
            int sh = se[t] + f.e - (sx.x + sy.x);
            sh = min(max(sh, 0), 127);
            acc += (unsigned __int128)(__int128)P << sh;
          }
        }
        __syncthreads();
      }
      if (valid) Cout[(size_t)sl * Yrows + y] = make_ulonglong2((unsigned long long)acc, (unsigned long long)(acc >> 64));
    }
  }
}

// ----------------------------------------------------------------- fixup ---
template <int FMT>
__global__ void __launch_bounds__(256) k_tc_fixup(GemmArgs a, const int4 *__restrict__ sta,
                                                  const int4 *__restrict__ stb, const int *__restrict__ slotA,
                                                  const int *__restrict__ slotB) {
  size_t n = (size_t)a.M * a.N;
  for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < n; o += (size_t)gridDim.x * blockDim.x) {
    int i = (int)(o / a.N), j = (int)(o % a.N);
    int4 ra = sta[i], rb = stb[j];
    if (!(ra.z && rb.z)) continue;
    if (tc_exact(ra, rb, slotA[i], slotB[j], a.K)) continue;
    slow_output<FMT>(a, i, j, a.out + (size_t)i * a.ldo + j,
                     a.quire ? a.quire + ((size_t)i * a.N + j) * a.nlimbs : nullptr);
  }
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

// [S][rows][Kp] int8 planes; box {128 (K), box_rows, S}; 128-byte swizzle.
int make_plane_map(CUtensorMap *m, void *base, int Kp, int rows, int S, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(kECuda, "quire_gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)S};
  cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)Kp * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)S};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kECuda, "quire_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return kOk;
}

inline size_t al(size_t v) { return (v + 255) / 256 * 256; }

struct TcLayout {
  int S, Kp, nkb, nchunks, capA, capB;
  size_t planesA, planesB, LA, LB, slotA, slotB, rowA, rowB, ctr, CA, CB, part, total;
};

// Correction buffers hold at most this many bytes per side; rows with a tail
// beyond the cap are finished by the fixup kernel instead.
constexpr size_t kCorrBudget = size_t(512) << 20;

TcLayout tc_layout(int fmt, int M, int N, int K) {
  TcLayout L{};
  L.S = fmt == 8 ? 3 : 4;
  L.Kp = (K + BK - 1) / BK * BK;
  L.nkb = L.Kp / BK;
  const int kbc = KCHUNK / BK;
  L.nchunks = (L.nkb + kbc - 1) / kbc;
  L.capA = (int)std::min<size_t>((size_t)M, std::max<size_t>(1, kCorrBudget / (16 * (size_t)std::max(N, 1))));
  L.capB = (int)std::min<size_t>((size_t)N, std::max<size_t>(1, kCorrBudget / (16 * (size_t)std::max(M, 1))));
  size_t o = 0;
  L.planesA = o; o += al((size_t)L.S * M * L.Kp);
  L.planesB = o; o += al((size_t)L.S * N * L.Kp);
  L.LA = o; o += al(4 * (size_t)M);
  L.LB = o; o += al(4 * (size_t)N);
  L.slotA = o; o += al(4 * (size_t)M);
  L.slotB = o; o += al(4 * (size_t)N);
  L.rowA = o; o += al(4 * (size_t)M);
  L.rowB = o; o += al(4 * (size_t)N);
  L.ctr = o; o += 256;
  L.CA = o; o += al(16 * (size_t)L.capA * N);
  L.CB = o; o += al(16 * (size_t)L.capB * M);
  L.part = o; o += L.nchunks > 1 ? al(16 * (size_t)L.nchunks * M * N) : 0;
  L.total = o;
  return L;
}

template <int S>
int launch_tc_gemm_kernel(const CUtensorMap &ma, const CUtensorMap &mb, const TcParams &p, cudaStream_t s) {
  using C = Cfg<S>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(k_quire_gemm_tc<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (attr_err != cudaSuccess)
    return set_error(kECuda, "quire_gemm: cannot set shared memory size: %s", cudaGetErrorString(attr_err));
  dim3 grid((p.N + C::BN - 1) / C::BN, (p.M + BM - 1) / BM, p.nchunks);
  if (grid.y > 65535u || grid.z > 65535u) return set_error(kERange, "quire_gemm: grid too large");
  k_quire_gemm_tc<S><<<grid, THREADS, C::SMEM, s>>>(ma, mb, p);
  return check_launch("quire_gemm_tc");
}

}  // namespace

bool gemm_tc_supported(int fmt, int M, int N, int K) {
  (void)fmt;
  return M > 0 && N > 0 && K > 0 && (size_t)K <= (size_t)1 << 30 && M <= 65535 * BM;
}

size_t gemm_tc_workspace(int fmt, int M, int N, int K) { return tc_layout(fmt, M, N, K).total; }

int launch_gemm_tc(const GemmArgs &a, const int4 *sta, const int4 *stb, void *ws, size_t ws_bytes, cudaStream_t s) {
  TcLayout L = tc_layout(a.fmt, a.M, a.N, a.K);
  if (ws_bytes < L.total) return set_error(kEWorkspace, "quire_gemm: tensor-core workspace too small");
  char *w = (char *)ws;
  int8_t *planesA = (int8_t *)(w + L.planesA), *planesB = (int8_t *)(w + L.planesB);
  int *LA = (int *)(w + L.LA), *LB = (int *)(w + L.LB);
  int *slotA = (int *)(w + L.slotA), *slotB = (int *)(w + L.slotB);
  int *rowA = (int *)(w + L.rowA), *rowB = (int *)(w + L.rowB);
  int *ctr = (int *)(w + L.ctr);
  ulonglong2 *CA = (ulonglong2 *)(w + L.CA), *CB = (ulonglong2 *)(w + L.CB);
  ulonglong2 *part = L.nchunks > 1 ? (ulonglong2 *)(w + L.part) : nullptr;

  cudaError_t e = cudaMemsetAsync(ctr, 0, 256, s);
  if (e != cudaSuccess) return set_error(kECuda, "quire_gemm: memset: %s", cudaGetErrorString(e));
  const int sms = sm_count();
  auto prep = [&](const void *codes, int rows, const int32_t *sc, const int4 *st, int8_t *planes, int *Lr,
                  int *slot, int *srow, int *counter, int cap) {
    long long blocks = ((long long)rows * 32 + 255) / 256;
    int g = (int)std::min<long long>(blocks, (long long)sms * 8);
    if (a.fmt == 8)
      k_tc_prep<8, 3><<<g, 256, 0, s>>>(codes, rows, a.K, L.Kp, sc, a.G, a.group, st, planes, Lr, slot, srow,
                                        counter, cap);
    else
      k_tc_prep<16, 4><<<g, 256, 0, s>>>(codes, rows, a.K, L.Kp, sc, a.G, a.group, st, planes, Lr, slot, srow,
                                         counter, cap);
    return check_launch("tc_prep");
  };
  int rc = prep(a.A, a.M, a.sa, sta, planesA, LA, slotA, rowA, ctr, L.capA);
  if (rc) return rc;
  rc = prep(a.B, a.N, a.sb, stb, planesB, LB, slotB, rowB, ctr + 1, L.capB);
  if (rc) return rc;

  // tail corrections (the kernels read the tail-row counts on the device)
  {
    dim3 ga((unsigned)std::min(L.capA, sms * 2), (unsigned)std::min((a.N + 255) / 256, 64));
    dim3 gb((unsigned)std::min(L.capB, sms * 2), (unsigned)std::min((a.M + 255) / 256, 64));
    if (a.fmt == 8) {
      k_tc_corr<8><<<ga, 256, 0, s>>>(a.A, a.B, a.N, a.K, a.sa, a.sb, a.G, a.group, sta, stb, LA, nullptr, rowA,
                                      ctr, L.capA, CA);
      rc = check_launch("tc_corr");
      if (rc) return rc;
      k_tc_corr<8><<<gb, 256, 0, s>>>(a.B, a.A, a.M, a.K, a.sb, a.sa, a.G, a.group, stb, sta, LB, LA, rowB,
                                      ctr + 1, L.capB, CB);
    } else {
      k_tc_corr<16><<<ga, 256, 0, s>>>(a.A, a.B, a.N, a.K, a.sa, a.sb, a.G, a.group, sta, stb, LA, nullptr, rowA,
                                       ctr, L.capA, CA);
      rc = check_launch("tc_corr");
      if (rc) return rc;
      k_tc_corr<16><<<gb, 256, 0, s>>>(a.B, a.A, a.M, a.K, a.sb, a.sa, a.G, a.group, stb, sta, LB, LA, rowB,
                                       ctr + 1, L.capB, CB);
    }
    rc = check_launch("tc_corr");
    if (rc) return rc;
  }

  int S = L.S;
  int bn = S == 3 ? Cfg<3>::BN : Cfg<4>::BN;
  CUtensorMap ma, mb;
  rc = make_plane_map(&ma, planesA, L.Kp, a.M, S, BM);
  if (rc) return rc;
  rc = make_plane_map(&mb, planesB, L.Kp, a.N, S, bn);
  if (rc) return rc;

  TcParams p{};
  p.M = a.M; p.N = a.N; p.K = a.K; p.Kp = L.Kp; p.nkb = L.nkb;
  p.kb_per_chunk = KCHUNK / BK; p.nchunks = L.nchunks;
  p.sta = sta; p.stb = stb; p.LA = LA; p.LB = LB; p.slotA = slotA; p.slotB = slotB;
  p.CA = CA; p.CB = CB;
  p.out = a.out; p.ldo = a.ldo; p.quire = a.quire; p.nlimbs = a.nlimbs; p.partial = part;
  rc = S == 3 ? launch_tc_gemm_kernel<3>(ma, mb, p, s) : launch_tc_gemm_kernel<4>(ma, mb, p, s);
  if (rc) return rc;
  size_t outs = (size_t)a.M * a.N;
  int g = (int)std::min<size_t>((outs + 255) / 256, (size_t)sms * 8);
  if (L.nchunks > 1) {
    k_tc_reduce<<<g, 256, 0, s>>>(p);
    rc = check_launch("tc_reduce");
    if (rc) return rc;
  }
  if (a.fmt == 8) k_tc_fixup<8><<<g, 256, 0, s>>>(a, sta, stb, slotA, slotB);
  else k_tc_fixup<16><<<g, 256, 0, s>>>(a, sta, stb, slotA, slotB);
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
