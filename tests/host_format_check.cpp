// host_format_check.cpp -- compiles the library's format logic
// (open-bposit_b200/csrc/bp_format.cuh, __host__ __device__ code) for the host
// and compares it with the CPU oracle (oracle/bposit_oracle.c) over every
// non-negative fp32 bit pattern (bp8 quantize, both modes), a strided sweep
// of all fp32 patterns (bp16 encode, both modes), every bp8 / bp16 code
// (decode) and random 128-bit magnitudes (bp32 round, its signed 64-bit form,
// and the bp16 round derived from it).  The streaming kernels' table-driven
// bp16 encoder and closed-form bp16 decoder, and the signed bp8 / bp16
// tables, are compared with the bit-string forms above over every fp32
// pattern and every bp16 code.  Test-only.
//
// usage: host_format_check <what> <threads>   what in q8 | e16 | e16t | signed | dec | bp32 | small
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <thread>
#include <vector>

#include "../open-bposit_b200/csrc/bp_format.cuh"

extern "C" {
void orc_quantize_bp8(const float *x, size_t n, int nearest, uint8_t *codes, float *values);
uint16_t orc_encode_bp16_one(float x, int rtne);
void orc_decode_me(int fmt_bits, uint32_t code, int64_t *mant, int *exp);
uint32_t orc_quire_to_bp32(const uint32_t *limbs, int nlimbs);
void orc_quire_to_bp16_batch(const uint32_t *limbs, int nlimbs, size_t n, uint16_t *out);
void orc_quantize_small(int nbits, const double *x, size_t n, uint8_t *codes);
}

static std::atomic<long long> g_bad{0};

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static void q8_range(uint64_t lo, uint64_t hi, bool nearest) {
  bp::QEntry tbl[256];
  for (int b = 0; b < 256; ++b) tbl[b] = bp::bp8_qentry(b, nearest);
  const size_t CH = 4096;
  float xs[CH];
  uint8_t ref[CH];
  long long bad = 0;
  for (uint64_t u0 = lo; u0 < hi; u0 += CH) {
    size_t n = (size_t)((hi - u0) < CH ? (hi - u0) : CH);
    for (size_t i = 0; i < n; ++i) xs[i] = f_of((uint32_t)(u0 + i));
    orc_quantize_bp8(xs, n, nearest ? 1 : 0, ref, nullptr);
    for (size_t i = 0; i < n; ++i) {
      uint32_t u = (uint32_t)(u0 + i);
      uint32_t a = u & 0x7FFFFFFFu;
      uint32_t code;
      if (a > 0x7F800000u) code = 0x80u;
      else {
        uint32_t mag = bp::bp8_apply(tbl[a >> 23], a & 0x7FFFFFu);
        code = (u >> 31) ? ((0u - mag) & 0xFFu) : mag;
      }
      if (code != ref[i]) {
        if (bad < 5) fprintf(stderr, "q8 mismatch nearest=%d x=%08x dev=%02x ref=%02x\n", nearest, u, code, ref[i]);
        ++bad;
      }
    }
  }
  g_bad += bad;
}

static void e16_range(uint64_t lo, uint64_t hi, uint64_t step, bool rtne) {
  long long bad = 0;
  for (uint64_t v = lo; v < hi; v += step) {
    uint32_t u = (uint32_t)v;
    uint32_t dev = bp::bp16_encode_bits(u, rtne);
    uint32_t ref = orc_encode_bp16_one(f_of(u), rtne ? 1 : 0);
    if (dev != ref) {
      if (bad < 5) fprintf(stderr, "e16 mismatch rtne=%d x=%08x dev=%04x ref=%04x\n", rtne, u, dev, ref);
      ++bad;
    }
  }
  g_bad += bad;
}

// the per-binade table encoder against bp16_encode_bits on [lo, hi)
static void e16t_range(uint64_t lo, uint64_t hi, bool rtne) {
  uint32_t tlo[256], thm[256];
  for (int b = 0; b < 256; ++b) bp::bp16_qentry(b, rtne, tlo[b], thm[b]);
  long long bad = 0;
  for (uint64_t v = lo; v < hi; ++v) {
    const uint32_t u = (uint32_t)v;
    const uint32_t b = (u >> 23) & 0xFFu;
    const uint32_t t = bp::bp16_encode_tbl(u, tlo[b], thm[b], rtne);
    const uint32_t ref = bp::bp16_encode_bits(u, rtne);
    if (t != ref) {
      if (bad < 5) fprintf(stderr, "e16t mismatch rtne=%d x=%08x tbl=%04x bits=%04x\n", rtne, u, t, ref);
      ++bad;
    }
  }
  g_bad += bad;
}

// the signed streaming tables against the per-binade forms on [lo, hi)
static void signed_range(uint64_t lo, uint64_t hi, int mode) {
  uint32_t x8[512], c8[512], x16[512], c16[512];
  for (int i = 0; i < 512; ++i) {
    bp::bp8_qentry_signed(i, mode == 1, x8[i], c8[i]);
    bp::bp16_qentry_signed(i, mode == 1, x16[i], c16[i]);
  }
  bp::QEntry t8[256];
  for (int b = 0; b < 256; ++b) t8[b] = bp::bp8_qentry(b, mode == 1);
  long long bad = 0;
  for (uint64_t v = lo; v < hi; ++v) {
    const uint32_t u = (uint32_t)v, a = u & 0x7FFFFFFFu, i = u >> 23;
    uint32_t r8;
    if (a > 0x7F800000u) r8 = 0x80u;
    else {
      const uint32_t mag = bp::bp8_apply(t8[a >> 23], a & 0x7FFFFFu);
      r8 = (u >> 31) ? ((0u - mag) & 0xFFu) : mag;
    }
    const uint32_t s8 = bp::bp8_encode_signed(u, x8[i], c8[i]);
    const uint32_t r16 = bp::bp16_encode_bits(u, mode == 1);
    const uint32_t s16 = mode == 1 ? bp::bp16_encode_signed<true>(u, x16[i], c16[i])
                                   : bp::bp16_encode_signed<false>(u, x16[i], c16[i]);
    if (s8 != r8 || s16 != r16) {
      if (bad < 5)
        fprintf(stderr, "signed mismatch mode=%d x=%08x bp8 %02x/%02x bp16 %04x/%04x\n", mode, u, s8, r8, s16, r16);
      ++bad;
    }
  }
  g_bad += bad;
}

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static uint64_t rnd() {
  rng_state ^= rng_state << 13; rng_state ^= rng_state >> 7; rng_state ^= rng_state << 17;
  return rng_state;
}

int main(int argc, char **argv) {
  const char *what = argc > 1 ? argv[1] : "q8";
  int nt = argc > 2 ? atoi(argv[2]) : 8;
  if (nt < 1) nt = 1;
  std::vector<std::thread> th;
  if (!strcmp(what, "q8")) {
    // every non-negative pattern and the negative half on a stride, both modes
    for (int mode = 0; mode < 2; ++mode) {
      for (int t = 0; t < nt; ++t) {
        uint64_t lo = (0x80000000ull * t) / nt, hi = (0x80000000ull * (t + 1)) / nt;
        th.emplace_back(q8_range, lo, hi, mode == 1);
      }
      for (auto &x : th) x.join();
      th.clear();
      for (uint64_t b = 0x80000000ull; b < 0x100000000ull; b += 0x01000000ull)
        q8_range(b, b + 0x4000, mode == 1);
    }
  } else if (!strcmp(what, "e16")) {
    for (int mode = 0; mode < 2; ++mode) {
      for (int t = 0; t < nt; ++t) {
        uint64_t lo = (0x100000000ull * t) / nt, hi = (0x100000000ull * (t + 1)) / nt;
        th.emplace_back(e16_range, lo, hi, 13, mode == 1);
      }
      for (auto &x : th) x.join();
      th.clear();
      // dense sweeps around every binade start and the bp16 range edges
      for (int b = 0; b < 256; ++b)
        for (uint32_t s = 0; s < 2; ++s) {
          uint64_t base = ((uint64_t)s << 31) | ((uint64_t)b << 23);
          e16_range(base, base + 0x2000, 1, mode == 1);
          e16_range(base + 0x7FFFFF - 0x2000, base + 0x800000, 1, mode == 1);
        }
    }
  } else if (!strcmp(what, "e16t")) {
    // every fp32 pattern, both modes
    for (int mode = 0; mode < 2; ++mode) {
      for (int t = 0; t < nt; ++t) {
        uint64_t lo = (0x100000000ull * t) / nt, hi = (0x100000000ull * (t + 1)) / nt;
        th.emplace_back(e16t_range, lo, hi, mode == 1);
      }
      for (auto &x : th) x.join();
      th.clear();
    }
  } else if (!strcmp(what, "signed")) {
    // every fp32 pattern, both modes: signed bp8 / bp16 tables vs the table / bit-string forms
    for (int mode = 0; mode < 2; ++mode) {
      for (int t = 0; t < nt; ++t) {
        uint64_t lo = (0x100000000ull * t) / nt, hi = (0x100000000ull * (t + 1)) / nt;
        th.emplace_back(signed_range, lo, hi, mode);
      }
      for (auto &x : th) x.join();
      th.clear();
    }
  } else if (!strcmp(what, "dec")) {
    long long bad = 0;
    for (uint32_t c = 0; c < 256; ++c) {
      int64_t m; int e; int dm, de;
      orc_decode_me(8, c, &m, &e);
      bp::posit_to_me<8, 2>(c, dm, de);
      if (m != dm || (m && e != de)) { ++bad; fprintf(stderr, "bp8 decode %02x\n", c); }
    }
    for (uint32_t c = 0; c < 65536; ++c) {
      int64_t m; int e; int dm, de;
      orc_decode_me(16, c, &m, &e);
      bp::posit_to_me<16, 3>(c, dm, de);
      if (m != dm || (m && e != de)) { if (bad < 5) fprintf(stderr, "bp16 decode %04x\n", c); ++bad; }
      // the closed-form fp32 decode of the streaming kernel
      if (bp::bp16_to_f32_bits(c) != bp::posit_to_f32_bits<16, 3>(c)) {
        if (bad < 5) fprintf(stderr, "bp16 f32 decode %04x\n", c);
        ++bad;
      }
    }
    g_bad += bad;
  } else if (!strcmp(what, "bp32")) {
    long long bad = 0;
    for (int it = 0; it < 2000000; ++it) {
      int bits = (int)(rnd() % 128) + 1;
      uint64_t hi = rnd(), lo = rnd();
      if (bits <= 64) { hi = 0; lo = bits == 64 ? lo : (lo & ((1ull << bits) - 1)); }
      else hi &= bits == 128 ? ~0ull : ((1ull << (bits - 64)) - 1);
      if (!hi && !lo) continue;
      int shift = (int)(rnd() % 200);     // quire bit of the magnitude's bit 0
      bool neg = rnd() & 1;
      if (bits + shift > 250) continue;
      // quire limbs: (mag << shift), negated if neg, 8 limbs
      uint32_t q[8] = {0};
      for (int i = 0; i < 128; ++i) {
        int bit = i < 64 ? (int)((lo >> i) & 1) : (int)((hi >> (i - 64)) & 1);
        if (bit) q[(i + shift) / 32] |= 1u << ((i + shift) % 32);
      }
      if (neg) {
        uint64_t c = 1;
        for (int i = 0; i < 8; ++i) { uint64_t s = (uint64_t)(uint32_t)~q[i] + c; q[i] = (uint32_t)s; c = s >> 32; }
      }
      uint32_t ref = orc_quire_to_bp32(q, 8);
      uint32_t dev = bp::bp32_from_mag(neg, hi, lo, shift - 96);
      if (ref != dev) { if (bad < 5) fprintf(stderr, "bp32 mismatch bits=%d shift=%d\n", bits, shift); ++bad; }
      if (bits <= 63) {   // the signed 64-bit form used for sums that fit int64
        const long long Q = neg ? -(long long)lo : (long long)lo;
        if (bp::bp32_from_i64(Q, shift - 96) != ref) {
          if (bad < 5) fprintf(stderr, "bp32 i64 mismatch bits=%d shift=%d\n", bits, shift);
          ++bad;
        }
      }
      // the bp16 round of the same quire, derived from the bp32 code
      uint16_t ref16;
      orc_quire_to_bp16_batch(q, 8, 1, &ref16);
      if (ref16 != bp::bp16_from_bp32(dev)) {
        if (bad < 5) fprintf(stderr, "bp16 mismatch bits=%d shift=%d\n", bits, shift);
        ++bad;
      }
    }
    // the direct value of a 64-bit sum (the finish kernel's fp32 hand-off)
    // against the value of its bposit32 code
    for (int it = 0; it < 2000000; ++it) {
      const int bits = (int)(rnd() % 63) + 1;
      const uint64_t mm = rnd() & ((1ull << bits) - 1);
      if (!mm) continue;
      const int L = (int)(rnd() % 601) - 300, extra = (int)(rnd() % 81) - 40;
      const long long Q = (rnd() & 1) ? -(long long)mm : (long long)mm;
      double v;
      if (!bp::bp32_value_i64(Q, L, extra, v)) continue;
      const uint32_t code = bp::bp32_from_i64(Q, L);
      bp::Dec d = bp::decode_posit<32, 3>(code);
      const double ref = (d.sign ? -1.0 : 1.0) * ldexp((double)((1u << d.fw) + d.fbits), d.scale - d.fw + extra);
      if (d.kind != 0 || v != ref) {
        if (bad < 5) fprintf(stderr, "bp32 value mismatch Q=%lld L=%d extra=%d\n", Q, L, extra);
        ++bad;
      }
    }
    // the 64-bit form against the 128-bit one over exponents past both ends
    // of the bposit32 range (minpos / maxpos saturation)
    for (int it = 0; it < 400000; ++it) {
      const int bits = (int)(rnd() % 63) + 1;
      const uint64_t m = bits == 64 ? rnd() : (rnd() & ((1ull << bits) - 1));
      if (!m) continue;
      const int L = (int)(rnd() % 801) - 400;
      const bool neg = rnd() & 1;
      const long long Q = neg ? -(long long)m : (long long)m;
      if (bp::bp32_from_i64(Q, L) != bp::bp32_from_mag(neg, 0u, m, L)) {
        if (bad < 5) fprintf(stderr, "bp32 i64 vs mag mismatch m=%llx L=%d\n", (unsigned long long)m, L);
        ++bad;
      }
    }
    g_bad += bad;
  } else if (!strcmp(what, "small")) {
    // bposit4 / AI-posit5 truncating encode: every fp32 pattern on a stride
    // (as double) plus random doubles around every binade in range
    long long bad = 0;
    std::vector<double> xs;
    for (uint64_t u = 0; u < 0x100000000ull; u += 4099) xs.push_back((double)f_of((uint32_t)u));
    for (int it = 0; it < 2000000; ++it) {
      int e = (int)(rnd() % 24) - 12;
      double m = 1.0 + (double)(rnd() >> 11) * 0x1p-53;
      double x = ldexp(m, e);
      if (rnd() & 1) x = -x;
      xs.push_back(x);
    }
    xs.push_back(0x1.5798ee2308c39p-28);
    xs.push_back(0x1.5798ee2308c3ap-28);
    std::vector<uint8_t> ref(xs.size());
    for (int nb = 4; nb <= 5; ++nb) {
      orc_quantize_small(nb, xs.data(), xs.size(), ref.data());
      for (size_t i = 0; i < xs.size(); ++i) {
        uint32_t dev = nb == 4 ? bp::small_encode<4, 1, 2>(xs[i]) : bp::small_encode<5, 1, 4>(xs[i]);
        if (dev != ref[i]) {
          if (bad < 5) fprintf(stderr, "small%d mismatch x=%a dev=%02x ref=%02x\n", nb, xs[i], dev, ref[i]);
          ++bad;
        }
      }
    }
    g_bad += bad;
  }
  printf("%s mismatches: %lld\n", what, (long long)g_bad.load());
  return g_bad.load() ? 1 : 0;
}
