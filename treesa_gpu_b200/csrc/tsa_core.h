// tsa_core.h -- arithmetic shared by the sm_100a kernels and the C++ host library of the B200 TreeSA
// annealer.  Everything here is bit-exact between host and device: integer hashing, the Philox stream,
// the integer-cost energy and the Metropolis test.
//
// Semantics follow the reference (xuanzhaogao/treesa_gpu):
//   * Philox4x32-10 with counter {v, sweep, chain, 0}            csrc/common.h:23-47
//   * par-order priorities  mix32 / par_pri                        csrc/common.h:250-263
//   * rule choice  pick_rule                                       csrc/common.h:233-238
//   * tc/sc energy of one move  energy_from_counts<0>              csrc/common.h:198-222
//   * Metropolis  u < expf(-beta*dE), u = (r >> 8) / 2^24          csrc/common.h:224-229
// The energy is evaluated from per-node cached (cost, size) words instead of seven popcounts per
// word: cost(v) = |z_v| + |x & y & ~z_v| is a property of node v alone, and a move at v changes the
// cost of exactly v and its pivot child, which the move itself computes.  Counts are exact integers,
// so the float energy is the same number the reference computes.
//
// expf: the reference's CPU port calls the host libm expf (glibc).  The device evaluates exp(x) in
// double with Tang's table-driven method (P. T. P. Tang, "Table-driven implementation of the
// exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2), 1989): x = (64n + j) ln2/64
// + r, exp(x) = 2^n 2^(j/64) p(r), |r| <= ln2/128, p the degree-6 Taylor polynomial.  Rounded once to
// float this is correctly rounded on every input checked; glibc's expf misrounds on ~1e5 negative
// inputs.  Those inputs and glibc's values are tabulated at build time (gen_expf_fixups.cpp); the
// table is consulted only when the uniform u falls within one ulp of exp(x), so the accept decision
// equals the host's on every input.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define TSA_HD __host__ __device__ __forceinline__
#define TSA_D __device__ __forceinline__
#else
#define TSA_HD inline
#endif

namespace tsa {

// ------------------------------------------------------------------------------------------------
// exact IEEE single/double operations (never contracted into FMAs, identical on host and device)
// ------------------------------------------------------------------------------------------------
TSA_HD float fadd(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fadd_rn(a, b);
#else
  volatile float r = a + b;
  return r;
#endif
}
TSA_HD float fsub(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fsub_rn(a, b);
#else
  volatile float r = a - b;
  return r;
#endif
}
TSA_HD float fmul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}

// ------------------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11).  One call per proposal.
// ------------------------------------------------------------------------------------------------
struct U4 {
  uint32_t x, y, z, w;
};

TSA_HD void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  // one 32x32->64 multiply (a single wide IMAD on the device)
  uint64_t p = (uint64_t)a * (uint64_t)b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

TSA_HD U4 philox10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int i = 0; i < 10; i++) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(0xD2511F53u, c0, hi0, lo0);
    mulhilo(0xCD9E8D57u, c2, hi1, lo1);
    uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return U4{c0, c1, c2, c3};
}

// ------------------------------------------------------------------------------------------------
// par-order priorities: 16-bit odd hash per (node, sweep, chain); 0 marks "visited".
// ------------------------------------------------------------------------------------------------
TSA_HD uint32_t mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}
// hash of the chain (once per chain) and of the sweep (once per sweep)
TSA_HD uint32_t chain_hash(uint32_t chain, uint32_t key0) { return mix32(chain ^ key0); }
TSA_HD uint32_t sweep_hash(uint32_t sweep, uint32_t hc) { return mix32(sweep * 0x85EBCA77u + hc); }
TSA_HD uint32_t node_pri(uint32_t v, uint32_t hs) { return (mix32(v * 0x9E3779B1u + hs) >> 16) | 1u; }
// par_band L (2..16): the band position of the node's depth d at the start of the sweep in the top four
// bits (the top of each band of L levels first), the node's own priority bits below; odd, never 0
// (csrc/common.h:264-268)
TSA_HD uint32_t band_pri(uint32_t pri, int d, int L) {
  return ((uint32_t)((L - 1 - d % L) & 15) << 12) | (pri & 0x0FFEu) | 1u;
}
// par_follow: priority of a follow-up visit of node v, even and nonzero (csrc/common.h:269-272)
TSA_HD uint32_t follow_pri(uint32_t v, uint32_t hs) {
  return ((mix32((v * 0x9E3779B1u + hs) ^ 0x5BD1E995u) >> 16) & 0xFFFEu) | 2u;
}
// a follow-up visit draws its own Philox stream: the sweep counter with its top bit set
TSA_HD uint32_t follow_sweep(uint32_t sweep) { return sweep | 0x80000000u; }

// Rule 0..3 (Julia rules 1..4) from the children kinds; -1 when both children are leaves.
TSA_HD int pick_rule(bool li, bool ri, uint32_t r) {
  if (li && ri) return (int)(r >> 30);
  if (li) return (int)(r >> 31);
  if (ri) return 2 + (int)(r >> 31);
  return -1;
}

// ------------------------------------------------------------------------------------------------
// Energy of one move from integer costs (tc mode).
//   costP/costV: cached costs of the pivot child and of v before the move,
//   sp, sd, sx: sizes of the pivot, of v and of the new pivot labels X,
//   cP1 = sx + |K & O & ~X|, cV1 = sd + |X & M & ~D|: costs after the move.
// ------------------------------------------------------------------------------------------------
struct EnergyParams {
  float sc_target, sc_weight;
  const float* lse_tab;  // 64 entries: log2(1 + 2^-d)
};

TSA_HD float lse_i(int a, int b, const float* tab) {
  int mx = a > b ? a : b;
  int d = a > b ? a - b : b - a;
  d = d < 63 ? d : 63;
  return fadd((float)mx, tab[d]);
}

TSA_HD float move_energy(int costP, int costV, int sp, int sd, int sx, int cP1, int cV1, float sc_target,
                         float sc_weight, const float* tab) {
  float tc0 = lse_i(costP, costV, tab);
  float tc1 = lse_i(cP1, cV1, tab);
  float dtc = fsub(tc1, tc0);
  int sc0 = sp > sd ? sp : sd;
  int sc1 = sx > sd ? sx : sd;
  int dsc = sc1 - sc0;
  int scmax = sc0 > sc1 ? sc0 : sc1;
  float w = ((float)scmax > sc_target) ? sc_weight : 0.0f;
  return fadd(fmul(w, (float)dsc), dtc);
}

// ------------------------------------------------------------------------------------------------
// expf by Tang's method in double precision, rounded once to float (x < 0 only).
// ------------------------------------------------------------------------------------------------
struct ExpConst {
  // ln2/64 split so that n*L1 is exact for |n| < 2^20; 64/ln2 rounded to double
  static constexpr double L1 = 0x1.62e42ff000000p-7;
  static constexpr double L2 = -0x1.718432a1b0e26p-41;
  static constexpr double INV = 0x1.71547652b82fep+6;
};

TSA_HD double dfma(double a, double b, double c) {
#ifdef __CUDA_ARCH__
  return __fma_rn(a, b, c);
#else
  return __builtin_fma(a, b, c);
#endif
}
TSA_HD double dmul(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(a, b);
#else
  volatile double r = a * b;
  return r;
#endif
}

// T[j] = 2^(j/64) rounded to double; table passed in so that host and device use their own copy.
TSA_HD float tang_expf(float xf, const double* T) {
  double x = (double)xf;
  if (x < -104.0) return 0.0f;  // exp(x) < 2^-150: rounds to +0
  double t = dmul(x, ExpConst::INV);
#ifdef __CUDA_ARCH__
  double nd = rint(t);
#else
  double nd = __builtin_rint(t);
#endif
  int n = (int)nd;
  double r = dfma(-nd, ExpConst::L1, x);
  r = dfma(-nd, ExpConst::L2, r);
  double p = 1.0 / 720.0;
  p = dfma(p, r, 1.0 / 120.0);
  p = dfma(p, r, 1.0 / 24.0);
  p = dfma(p, r, 1.0 / 6.0);
  p = dfma(p, r, 0.5);
  p = dfma(p, r, 1.0);
  p = dfma(p, r, 1.0);
  int j = n & 63, k = n >> 6;  // arithmetic shift: floor(n / 64)
  double y = dmul(T[j], p);
  // exact scaling by 2^k (k in [-163, 0]: a normal double)
  uint64_t bits = (uint64_t)(int64_t)(1023 + k) << 52;
  double s;
#ifdef __CUDA_ARCH__
  s = __longlong_as_double((long long)bits);
#else
  __builtin_memcpy(&s, &bits, 8);
#endif
  y = dmul(y, s);
  return (float)y;
}

// float bits helpers
TSA_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}
TSA_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

// glibc's expf value at x if x is in the fix-up table (sorted by the bit pattern of x), else e.
TSA_HD float fixup_lookup(float x, float e, const uint32_t* fx, const uint32_t* fg, int nfix) {
  uint32_t key = f2u(x);
  int lo = 0, hi = nfix;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    uint32_t v = fx[mid];
    if (v < key) lo = mid + 1;
    else hi = mid;
  }
  if (lo < nfix && fx[lo] == key) return u2f(fg[lo]);
  return e;
}

// Exact decision u < expf(x) for x < 0 (glibc expf): Tang's correctly rounded value plus the table.
TSA_HD bool metropolis_exact(float u, float x, const double* T, const uint32_t* fx, const uint32_t* fg, int nfix) {
  float e = tang_expf(x, T);
  // glibc's value differs from e by at most one ulp; only a u next to e can see the difference
  uint32_t eb = f2u(e);
  float lo = eb ? u2f(eb - 1u) : 0.0f;  // previous float (e >= +0)
  if (u < lo) return true;
  float hi = u2f(eb + 1u);
  if (u >= hi) return false;
  float g = fixup_lookup(x, e, fx, fg, nfix);
  return u < g;
}

#ifdef __CUDACC__
// 2^t by the SFU (ex2.approx.f32: relative error about 2^-22 on the whole range)
__device__ __forceinline__ float ex2_approx(float t) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}
#endif

// Metropolis test identical to the host's  u < expf(-beta * dE)  (glibc expf).  The device first
// decides with a single-instruction 2^(x log2 e); only when u lies within a relative margin of 8e-6 of
// that value (6x the worst error of the approximation for -17.5 < x < 0, checked exhaustively on the
// GPU by tests/test_gpu_metropolis.py) does it evaluate the exact value.  Below x = -17.5, exp(x) is
// below the smallest nonzero u (2^-24), so only u = 0 can be accepted.
TSA_HD bool metropolis(uint32_t r, float beta, float dE, const double* T, const uint32_t* fx, const uint32_t* fg,
                       int nfix) {
  float u = (float)(r >> 8) * (1.0f / 16777216.0f);
  float x = fmul(-beta, dE);
  if (!(x < 0.0f)) return true;  // expf(x) >= 1 > u
#ifdef __CUDA_ARCH__
  if (x >= -17.5f) {
    float ea = ex2_approx(__fmul_rn(x, 1.44269504088896341f));
    if (u < __fmul_rn(ea, 1.0f - 8e-6f)) return true;
    if (u > __fmul_rn(ea, 1.0f + 8e-6f)) return false;
  } else if (r >> 8) {
    return false;  // u >= 2^-24 > exp(x)
  }
#endif
  return metropolis_exact(u, x, T, fx, fg, nfix);
}

}  // namespace tsa
