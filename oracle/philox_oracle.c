/*
 * CPU restatement of the reference's initial-noise stream -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker for libltxb200's Philox kernel: only tests/, smoke() and
 * bench.py's cpu_baseline leg may load it. The product path never calls it.
 *
 * What it restates:
 *  - Philox4x32-10, the counter-based cipher of Salmon, Moraes, Dror and Shaw,
 *    "Parallel random numbers: as easy as 1, 2, 3" (SC'11): 10 rounds of two 32x32->64
 *    multiplies (constants 0xD2511F53, 0xCD9E8D57) with a Weyl key schedule
 *    (0x9E3779B9, 0xBB67AE85), all published in that paper.
 *  - torch's grid-stride normal fill as the reference drives it
 *    (lipaul/ltx-nv cuda_c_standalone/common/philox.cu:6-35): thread idx of
 *    threads = 256*grid uses counter (offset/4 + round, subsequence idx), key = seed;
 *    round r's four normals go to out[r*4*threads + ii*threads + idx].
 *  - The normal transform as the textbook Box-Muller method, evaluated in double
 *    precision: u = (x + 0.5) / 2^32, v likewise, r = sqrt(-2 ln u),
 *    (n0, n1) = (r sin 2 pi v, r cos 2 pi v) for the word pairs (x0, x1), (x2, x3).
 *    The pairing/order convention was fixed against the reference's golden noise
 *    (cuda_c_standalone/artifacts/m1_philox/*.bin); being evaluated in double rather
 *    than in the GPU's single precision, it matches the reference's bf16 values except
 *    for rare 1-ulp rounding ties.
 */
#include <math.h>
#include <stdint.h>

#define PHILOX_M0 0xD2511F53u
#define PHILOX_M1 0xCD9E8D57u
#define PHILOX_W0 0x9E3779B9u
#define PHILOX_W1 0xBB67AE85u

void oracle_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = (uint64_t)PHILOX_M0 * c0;
    const uint64_t p1 = (uint64_t)PHILOX_M1 * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += PHILOX_W0;
    k1 += PHILOX_W1;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

static void block_for(uint64_t seed, uint64_t subseq, uint64_t ctr, uint32_t out[4]) {
  const uint32_t c[4] = {(uint32_t)ctr, (uint32_t)(ctr >> 32), (uint32_t)subseq, (uint32_t)(subseq >> 32)};
  const uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  oracle_philox4x32_10(c, k, out);
}

/* Raw words: out[(r*threads + t)*4 + j] = word j of counter (offset/4 + r, t). */
void oracle_philox_raw(uint32_t* out, int64_t threads, int64_t rounds, uint64_t seed, uint64_t offset) {
  for (int64_t r = 0; r < rounds; ++r)
    for (int64_t t = 0; t < threads; ++t) block_for(seed, (uint64_t)t, offset / 4 + (uint64_t)r, out + (r * threads + t) * 4);
}

static void box_muller(uint32_t x, uint32_t y, double* a, double* b) {
  const double two32 = 4294967296.0;
  const double u = ((double)x + 0.5) / two32;
  const double v = ((double)y + 0.5) / two32;
  const double r = sqrt(-2.0 * log(u));
  const double th = 2.0 * M_PI * v;
  *a = r * sin(th);
  *b = r * cos(th);
}

/* Normal fill of n elements exactly as the grid-stride kernel lays it out. */
void oracle_randn(double* out, int64_t n, uint64_t seed, uint64_t offset, int grid) {
  const int64_t threads = (int64_t)grid * 256;
  const int64_t step = threads * 4;
  const int64_t rounds = (n - 1) / step + 1;
  for (int64_t r = 0; r < rounds; ++r) {
    for (int64_t t = 0; t < threads; ++t) {
      const int64_t base = r * step + t;
      if (base >= n) break;
      uint32_t w[4];
      block_for(seed, (uint64_t)t, offset / 4 + (uint64_t)r, w);
      double v[4];
      box_muller(w[0], w[1], &v[0], &v[1]);
      box_muller(w[2], w[3], &v[2], &v[3]);
      for (int ii = 0; ii < 4; ++ii) {
        const int64_t li = base + ii * threads;
        if (li < n) out[li] = v[ii];
      }
    }
  }
}

/* Generator bookkeeping (philox.cu:6-17): grid from the launch policy, offset advance. */
int64_t oracle_philox_grid(int64_t n, int sms, int max_threads_per_sm) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)sms * (max_threads_per_sm / 256);
  return g < cap ? g : cap;
}

int64_t oracle_philox_offset_increment(int64_t n, int grid) {
  return ((n - 1) / ((int64_t)256 * grid * 4) + 1) * 4;
}
