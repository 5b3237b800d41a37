// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.  Drives the reference's own CPU port, csrc/cpu_ref.h
// (ref_par_sweep<0>, ref_optimize_subtree<0>) with csrc/common.h, compiled from the reference's source
// tree by oracle/Makefile (-I <reference>/csrc) into oracle/_ref/libtsa_cpuref.so.  Nothing from the
// reference is copied here: this file only supplies what the reference's host code (csrc/treesa_gpu.cu)
// supplies around those headers -- the lse table definition (:52, filled as at :2075), the Philox key
// (splitmix64 of the seed, :1408-1413, :1457-1459), the RefTree built from a chain record (:2012-2028)
// and the sweep ids lev*niters+it (:2029-2039).
//
// Used by tests (bit-exactness of oracle/tsa_oracle.cpp and of the CUDA path against the reference
// itself) and by bench.py's reference arm / cpu_baseline (timed on the host cores).
#include <omp.h>
#include <stdint.h>
#include <string.h>

#include <chrono>
#include <cmath>
#include <vector>

#include "cpu_ref.h"

float h_lse_tab[64];

namespace {
uint64_t splitmix64_h(uint64_t x) {
  x += 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}
void fill_table() {
  for (int d = 0; d < 64; d++) h_lse_tab[d] = (float)std::log2(1.0 + std::exp2(-(double)d));
}
}  // namespace

extern "C" {

// Chains c0..c0+nch-1 from trees_in / labels_in ([nch][m-1] words, [nch][m-1][nw64] u64 bitsets of
// the internal nodes' output labels) and slice sets S_in ([nch][nw64] or NULL), nbetas levels of
// niters sweeps each; order 0 = par, 1 = preorder.  Writes trees_out / labels_out (labels_out may be
// NULL); counters = {proposals, accepts}; par_band / par_follow as the CLI's --par-band / --par-follow
// (treesa_gpu.cu:1388-1389, 1524-1527); mode 0 tc, 1 gpu model, 2 h100 model (default constants);
// returns the seconds spent in the sweep loops.
double ref_sweeps(int m, int nlab, const int* ix_off, const int* ix_lab, int order, uint64_t seed, double sc_target,
                  double sc_weight, const float* betas, int nbetas, int niters, int nch, int c0,
                  const uint32_t* trees_in, const uint64_t* labels_in, const uint64_t* S_in, uint32_t* trees_out,
                  uint64_t* labels_out, long long* counters, int nthreads, int par_band, int par_follow, int mode) {
  fill_table();
  const int nw = (nlab + 63) / 64 > 0 ? (nlab + 63) / 64 : 1, nint = m - 1;
  Params P{};
  P.m = m;
  P.nint = nint;
  P.sc_target = (float)sc_target;
  P.sc_weight = (float)sc_weight;
  P.par_band = par_band;
  P.par_follow = par_follow;
  // the default gpu / h100 model constants, as the reference's Runner sets Params from them
  // (treesa_gpu.cu:1460-1475, defaults of treesa_gpu/driver.py / trees.py)
  {
    const double gm[6] = {11.9e15, 1.6e13, 6, 6, 8, 4e-6};
    const double hm[9] = {4e-6, 1.23e13, 5.44e-14, 7.68e-15, 6.37e-14, 2.02e-16, 1.77e-13, 14, 1e-12};
    P.lpeak = (float)std::log2(gm[0]);
    P.lbw = (float)std::log2(gm[1]);
    P.m0 = (int)gm[2];
    P.n0 = (int)gm[3];
    P.k0 = (int)gm[4];
    P.llaunch = (float)std::log2(gm[5]);
    P.v2_l3launch = (float)std::log2(3 * hm[0]);
    P.v2_lperm2 = (float)std::log2(2 / hm[1]);
    P.v2_lcc_bit = (float)std::log2(hm[2]);
    P.v2_lcc_cell = (float)std::log2(hm[3]);
    P.v2_ltc_bit = (float)std::log2(hm[4]);
    P.v2_ltc_pad = (float)std::log2(hm[5]);
    P.v2_ltc_out = (float)std::log2(hm[6]);
    P.v2_small_rank = (int)hm[7];
    P.v2_lsmall_cell = (float)std::log2(hm[8]);
  }
  uint64_t k = splitmix64_h(seed);
  P.key0 = (uint32_t)k;
  P.key1 = (uint32_t)(k >> 32);
  if (nthreads > 0) omp_set_num_threads(nthreads);
  long long np = 0, na = 0;
  double secs = 0;
#pragma omp parallel reduction(+ : np, na) reduction(max : secs)
  {
#pragma omp for schedule(dynamic, 1)
    for (int q = 0; q < nch; q++) {
      RefTree T;
      T.m = m;
      T.left.assign(2 * m - 1, -1);
      T.right.assign(2 * m - 1, -1);
      T.labels.resize(2 * m - 1);
      T.sliced.assign(nlab > 0 ? nlab : 1, 0);
      if (S_in)
        for (int l = 0; l < nlab; l++) T.sliced[l] = (char)(S_in[(size_t)q * nw + (l >> 6)] >> (l & 63) & 1ull);
      for (int i = 0; i < m; i++) {
        T.labels[i].assign(ix_lab + ix_off[i], ix_lab + ix_off[i + 1]);
        std::sort(T.labels[i].begin(), T.labels[i].end());
      }
      const uint32_t* tr = trees_in + (size_t)q * nint;
      const uint64_t* lb = labels_in + (size_t)q * nint * nw;
      for (int i = 0; i < nint; i++) {
        T.left[m + i] = (int)(tr[i] & 0xFFFFu);
        T.right[m + i] = (int)(tr[i] >> 16);
        for (int l = 0; l < nlab; l++)
          if (lb[(size_t)i * nw + (l >> 6)] >> (l & 63) & 1ull) T.labels[m + i].push_back(l);
      }
      long long a = 0, b = 0;
      auto t0 = std::chrono::steady_clock::now();
      for (int lev = 0; lev < nbetas; lev++)
        for (int it = 0; it < niters; it++) {
          uint32_t sw = (uint32_t)(lev * niters + it);
          const uint32_t ch = (uint32_t)(c0 + q);
          if (order == 0) {
            if (mode == 1) ref_par_sweep<1>(T, betas[lev], sw, ch, P, a, b);
            else if (mode == 2) ref_par_sweep<2>(T, betas[lev], sw, ch, P, a, b);
            else ref_par_sweep<0>(T, betas[lev], sw, ch, P, a, b);
          } else {
            if (mode == 1) ref_optimize_subtree<1>(T, 2 * m - 2, betas[lev], sw, ch, P, a, b);
            else if (mode == 2) ref_optimize_subtree<2>(T, 2 * m - 2, betas[lev], sw, ch, P, a, b);
            else ref_optimize_subtree<0>(T, 2 * m - 2, betas[lev], sw, ch, P, a, b);
          }
        }
      double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      secs = dt > secs ? dt : secs;
      np += a;
      na += b;
      uint32_t* to = trees_out + (size_t)q * nint;
      for (int i = 0; i < nint; i++) to[i] = (uint32_t)T.left[m + i] | ((uint32_t)T.right[m + i] << 16);
      if (labels_out) {
        uint64_t* lo = labels_out + (size_t)q * nint * nw;
        memset(lo, 0, (size_t)nint * nw * 8);
        for (int i = 0; i < nint; i++)
          for (int l : T.labels[m + i]) lo[(size_t)i * nw + (l >> 6)] |= 1ull << (l & 63);
      }
    }
  }
  if (counters) counters[0] = np, counters[1] = na;
  return secs;
}

int ref_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
