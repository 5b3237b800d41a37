// tsa_oracle.cpp -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference TreeSA annealing path
// (xuanzhaogao/treesa_gpu), used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
// as the checker of the CUDA path.  The product (treesa_gpu_b200) never links, loads or calls it.
//
// Written in C-style C++ so that the population steps can call the same standard-library algorithms
// the reference calls (std::mt19937_64, std::uniform_real_distribution<double>, std::sort): their
// libstdc++ behaviour is part of the reference's semantics.  Label sets are packed u64 bitsets and
// every move recounts the label sets it reads (no cached costs): an independent restatement of
// csrc/cpu_ref.h, not a copy of the GPU path.
//
// Parity status: pinned.  tests/test_oracle.py checks this file bit for bit against the reference's own
// cpu_ref.h compiled from its sources (oracle/_ref, recipe oracle/Makefile) and against the golden
// values of the reference's logs (tests/golden/).
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <functional>
#include <numeric>
#include <random>
#include <vector>

#include "../include/treesa_b200.h"

namespace {

// ---------------------------------------------------------------------------------------------
// RNG and hashing (csrc/common.h:23-47, csrc/common.h:250-263, csrc/treesa_gpu.cu:1408-1413)
// ---------------------------------------------------------------------------------------------
uint64_t splitmix64(uint64_t x) {  // treesa_gpu.cu:1408-1413
  x += 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}

struct R4 {
  uint32_t a, b, c, d;
};
R4 philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {  // common.h:36-47
  for (int i = 0; i < 10; i++) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c0 = n0, c1 = n1, c2 = n2, c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return R4{c0, c1, c2, c3};
}

uint32_t mix32(uint32_t h) {  // common.h:250-257
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}
uint32_t par_pri(uint32_t v, uint32_t s, uint32_t c, uint32_t key0) {  // common.h:260-263
  uint32_t h = mix32(v * 0x9E3779B1u + mix32(s * 0x85EBCA77u + mix32(c ^ key0)));
  return (h >> 16) | 1u;
}
// par_band L: band position of the depth d at the start of the sweep, then the node's own bits (common.h:264-268)
uint32_t par_band_pri(uint32_t v, uint32_t s, uint32_t c, uint32_t key0, int d, int L) {
  return ((uint32_t)((L - 1 - d % L) & 15) << 12) | (par_pri(v, s, c, key0) & 0x0FFEu) | 1u;
}
// par_follow: even priority of a follow-up visit; hs = mix32(s * 0x85EBCA77 + mix32(c ^ key0)) (common.h:269-272)
uint32_t par_follow_pri(uint32_t v, uint32_t hs) {
  return ((mix32((v * 0x9E3779B1u + hs) ^ 0x5BD1E995u) >> 16) & 0xFFFEu) | 2u;
}

int pick_rule(bool li, bool ri, uint32_t r) {  // common.h:233-238
  if (li && ri) return (int)(r >> 30);
  if (li) return (int)(r >> 31);
  if (ri) return 2 + (int)(r >> 31);
  return -1;
}

// ---------------------------------------------------------------------------------------------
// Energy arithmetic (csrc/common.h:96-126, 198-229; table filled as at csrc/treesa_gpu.cu:2075)
// ---------------------------------------------------------------------------------------------
struct Table {
  float t[64];
  Table() {
    for (int d = 0; d < 64; d++) t[d] = (float)log2(1.0 + exp2(-(double)d));
  }
};
const Table& lse_table() {
  static const Table T;
  return T;
}
float lse_i(int a, int b) {  // common.h:114-118
  int mx = a > b ? a : b, d = a > b ? a - b : b - a;
  volatile float r = (float)mx + lse_table().t[d < 63 ? d : 63];
  return r;
}
float lse_f(float a, float b) {  // common.h:121-126
  float mx = a > b ? a : b, mn = a > b ? b : a;
  if (mx == -INFINITY) return mx;
  volatile float one = 1.0f + exp2f(mn - mx);
  volatile float r = mx + log2f(one);
  return r;
}
bool metropolis(uint32_t r, float beta, float dE) {  // common.h:226-229 (host libm expf)
  float u = (float)(r >> 8) * (1.0f / 16777216.0f);
  volatile float x = -beta * dE;
  return u < expf(x);
}

// ---------------------------------------------------------------------------------------------
// Instance, bitsets, trees
// ---------------------------------------------------------------------------------------------
struct Inst {  // read_instance, treesa_gpu.cu:1035-1073
  int m = 0, nlab = 0, nw = 0;
  std::vector<std::vector<int>> ixs;
  std::vector<int> iy, total;
  std::vector<char> in_iy;
  std::vector<uint64_t> leaf;  // [m][nw]
};

bool load_instance(const tsa_instance* I, Inst& S, char* err, size_t errlen) {
  if (!I || I->m < 3 || I->nlab < 0 || 2 * I->m - 1 > 65535) {
    snprintf(err, errlen, "oracle: need 3 <= m and 2m-1 <= 65535");
    return false;
  }
  S.m = I->m;
  S.nlab = I->nlab;
  S.nw = (I->nlab + 63) / 64;
  if (S.nw == 0) S.nw = 1;
  S.ixs.resize(S.m);
  S.total.assign(S.nlab, 0);
  S.in_iy.assign(S.nlab, 0);
  for (int i = 0; i < S.m; i++) {
    for (int k = I->ix_offsets[i]; k < I->ix_offsets[i + 1]; k++) S.ixs[i].push_back(I->ix_labels[k]);
    std::sort(S.ixs[i].begin(), S.ixs[i].end());
    if (std::adjacent_find(S.ixs[i].begin(), S.ixs[i].end()) != S.ixs[i].end()) {
      snprintf(err, errlen, "oracle: repeated label inside one tensor");
      return false;
    }
    for (int l : S.ixs[i]) {
      if (l < 0 || l >= S.nlab) {
        snprintf(err, errlen, "oracle: label out of range");
        return false;
      }
      S.total[l]++;
    }
  }
  for (int j = 0; j < I->niy; j++) {
    if (I->iy[j] < 0 || I->iy[j] >= S.nlab) {
      snprintf(err, errlen, "oracle: open label out of range");
      return false;
    }
    S.iy.push_back(I->iy[j]);
    S.in_iy[I->iy[j]] = 1;
  }
  S.leaf.assign((size_t)S.m * S.nw, 0);
  for (int i = 0; i < S.m; i++)
    for (int l : S.ixs[i]) S.leaf[(size_t)i * S.nw + (l >> 6)] |= 1ull << (l & 63);
  return true;
}

// A chain: children words of internal nodes, unsliced output-label bitsets, slice set.
struct Chain {
  std::vector<uint32_t> ch;   // [m-1]
  std::vector<uint64_t> lab;  // [m-1][nw]
  std::vector<uint64_t> S;    // [nw]
};

// random_exprtree, treesa_gpu.cu:1101-1123 (post-order numbering from m, root 2m-2)
std::vector<uint32_t> random_tree(int m, uint64_t seed) {
  std::mt19937_64 rng(seed);
  std::vector<uint32_t> ch(m - 1);
  int next = m;
  std::function<int(const std::vector<int>&)> build = [&](const std::vector<int>& xs) -> int {
    int n = (int)xs.size();
    if (n == 1) return xs[0];
    std::vector<char> mask(n);
    int cnt = 0;
    for (int i = 0; i < n; i++) {
      mask[i] = (char)(rng() & 1);
      cnt += mask[i];
    }
    if (cnt == 0 || cnt == n) {
      int i = (int)(rng() % n);
      mask[i] = !mask[i];
    }
    std::vector<int> a, b;
    for (int i = 0; i < n; i++) (mask[i] ? a : b).push_back(xs[i]);
    int l = build(a), r = build(b);
    int v = next++;
    ch[v - m] = (uint32_t)l | ((uint32_t)r << 16);
    return v;
  };
  std::vector<int> all(m);
  std::iota(all.begin(), all.end(), 0);
  build(all);
  return ch;
}

// preorder + validity, treesa_gpu.cu:1127-1145
bool preorder(int m, const uint32_t* ch, std::vector<int>& order) {
  order.clear();
  std::vector<char> seen(2 * m - 1, 0);
  std::vector<int> st{2 * m - 2};
  int nseen = 0;
  while (!st.empty()) {
    int v = st.back();
    st.pop_back();
    if (v < 0 || v >= 2 * m - 1 || seen[v]) return false;
    seen[v] = 1;
    nseen++;
    if (v >= m) {
      order.push_back(v);
      st.push_back((int)(ch[v - m] >> 16));
      st.push_back((int)(ch[v - m] & 0xFFFFu));
    }
  }
  return nseen == 2 * m - 1;
}

// labels_from_topology, treesa_gpu.cu:1149-1172: label l is an output of v iff it occurs in v's
// subtree and (also outside it, or is open)
bool labels_from_topology(const Inst& I, const uint32_t* ch, uint64_t* lab) {
  const int m = I.m, L = I.nlab, nw = I.nw;
  std::vector<int> order;
  if (!preorder(m, ch, order)) return false;
  std::vector<uint16_t> cnt((size_t)(m - 1) * std::max(L, 1), 0);
  for (int k = (int)order.size() - 1; k >= 0; k--) {
    int v = order[k];
    uint16_t* cv = &cnt[(size_t)(v - m) * L];
    for (int side = 0; side < 2; side++) {
      int u = side ? (int)(ch[v - m] >> 16) : (int)(ch[v - m] & 0xFFFFu);
      if (u < m) {
        for (int l : I.ixs[u]) cv[l]++;
      } else {
        const uint16_t* cu = &cnt[(size_t)(u - m) * L];
        for (int l = 0; l < L; l++) cv[l] += cu[l];
      }
    }
    uint64_t* z = lab + (size_t)(v - m) * nw;
    for (int w = 0; w < nw; w++) z[w] = 0;
    for (int l = 0; l < L; l++)
      if (cv[l] > 0 && (cv[l] < I.total[l] || I.in_iy[l])) z[l >> 6] |= 1ull << (l & 63);
  }
  return true;
}

struct Models {
  float lpeak, lbw, llaunch;
  int m0, n0, k0;
  float l3launch, lperm2, lcc_bit, lcc_cell, ltc_bit, ltc_pad, ltc_out, lsmall_cell;
  int small_rank;
};
Models make_models(const double* gm_in, const double* hm_in) {  // Runner ctor, treesa_gpu.cu:1461-1475
  const double gm_def[6] = {11.9e15, 1.6e13, 6, 6, 8, 4e-6};
  const double hm_def[9] = {4e-6, 1.23e13, 5.44e-14, 7.68e-15, 6.37e-14, 2.02e-16, 1.77e-13, 14, 1e-12};
  const double* gm = gm_in ? gm_in : gm_def;
  const double* hm = hm_in ? hm_in : hm_def;
  Models M;
  M.lpeak = (float)log2(gm[0]);
  M.lbw = (float)log2(gm[1]);
  M.m0 = (int)gm[2], M.n0 = (int)gm[3], M.k0 = (int)gm[4];
  M.llaunch = (float)log2(gm[5]);
  M.l3launch = (float)log2(3 * hm[0]);
  M.lperm2 = (float)log2(2 / hm[1]);
  M.lcc_bit = (float)log2(hm[2]);
  M.lcc_cell = (float)log2(hm[3]);
  M.ltc_bit = (float)log2(hm[4]);
  M.ltc_pad = (float)log2(hm[5]);
  M.ltc_out = (float)log2(hm[6]);
  M.small_rank = (int)hm[7];
  M.lsmall_cell = (float)log2(hm[8]);
  return M;
}
// Log-domain model costs of one pairwise contraction with label counts B, M, N, K (common.h:128-152),
// float with the host libm's log2f/exp2f through lse_f, as the reference's CPU port evaluates them.
float gpu_lt(int B, int M, int N, int K, const Models& P) {
  int Me = M > P.m0 ? M : P.m0, Ne = N > P.n0 ? N : P.n0, Ke = K > P.k0 ? K : P.k0;
  volatile float lops = (float)(1 + B + Me + Ne + Ke) - P.lpeak;
  volatile float lbits = lse_f(lse_f((float)(B + M + K), (float)(B + N + K)), (float)(B + M + N)) - P.lbw;
  float lt = lops > lbits ? lops : lbits;
  return lse_f(lt, P.llaunch);
}
float h100_lt(int B, int M, int N, int K, const Models& P) {
  if (B + M + N <= P.small_rank) {
    volatile float r = P.lsmall_cell + (float)(B + M + N + K);
    return r;
  }
  float la = (float)(B + M + K), lb = (float)(B + N + K), lc = (float)(B + M + N);
  float lab = lse_f(la, lb), lmoved = lse_f(lab, lc);
  volatile float perm = P.lperm2 + lab;
  volatile float cb = P.lcc_bit + lmoved, cc = P.lcc_cell + (float)(B + M + N + K);
  float best = lse_f(cb, cc);
  int MN = M > N ? M : N;
  if (K >= 7 && MN >= 5) {
    int Me = M > 6 ? M : 6, Ne = N > 6 ? N : 6, Ke = K > 8 ? K : 8;
    volatile float tb = P.ltc_bit + lmoved, tp = P.ltc_pad + (float)(B + Me + Ne + Ke), to = P.ltc_out + lc;
    float tc = lse_f(lse_f(tb, tp), to);
    best = tc < best ? tc : best;
  }
  return lse_f(lse_f(P.l3launch, perm), best);
}
// count3 of common.h:172-177 on one masked word: x, y -> z
inline void count3(uint64_t x, uint64_t y, uint64_t z, int& B, int& M, int& N, int& K) {
  B += __builtin_popcountll(x & y & z);
  M += __builtin_popcountll(x & ~y & z);
  N += __builtin_popcountll(~x & y & z);
  K += __builtin_popcountll(x & y & ~z);
}

struct Par {
  int m, nint, nw, leaf_sc, slicing, slice_moves, slice_every, max_slices;
  float sc_target, sc_weight;
  uint32_t key0, key1;
  int par_band, par_follow;  // par-order variants (off: 0)
  int mode;                  // energy: 0 tc, 1 gpu model, 2 h100 model
  Models mo;
};
// log2 cost of the contraction (x, y) -> z in mode 1 or 2 (node_cost, common.h:158-162)
inline float model_cost(const Par& P, int B, int M, int N, int K) {
  return P.mode == 1 ? gpu_lt(B, M, N, K, P.mo) : h100_lt(B, M, N, K, P.mo);
}

inline const uint64_t* set_of(const Inst& I, const Chain& C, int v) {
  return v < I.m ? &I.leaf[(size_t)v * I.nw] : &C.lab[(size_t)(v - I.m) * I.nw];
}
inline int popc(uint64_t x) { return __builtin_popcountll(x); }

// ---------------------------------------------------------------------------------------------
// One TreeSA proposal at internal node v: csrc/cpu_ref.h:89-121 (rules 1..4 of Julia
// optimize_subtree!, rw_weight 0), label sets as bitsets masked by ~S.
// Returns true if a proposal was made.
// ---------------------------------------------------------------------------------------------
bool visit(const Inst& I, const Par& P, Chain& C, int v, float beta, uint32_t sweep, uint32_t chain,
           long long& nprop, long long& nacc) {
  const int m = I.m, nw = I.nw;
  uint32_t cw = C.ch[v - m];
  int L = (int)(cw & 0xFFFFu), R = (int)(cw >> 16);
  bool li = L >= m, ri = R >= m;
  if (!li && !ri) return false;
  R4 rnd = philox((uint32_t)v, sweep, chain, 0u, P.key0, P.key1);
  int rule = pick_rule(li, ri, rnd.a) + 1;
  // a, b: children of the pivot (a stays, b moves up); ab: the pivot; c: the other child
  int a, b, ab, c;
  uint32_t cL = li ? C.ch[L - m] : 0, cR = ri ? C.ch[R - m] : 0;
  if (rule == 1) { a = (int)(cL & 0xFFFFu); b = (int)(cL >> 16); ab = L; c = R; }
  else if (rule == 2) { a = (int)(cL >> 16); b = (int)(cL & 0xFFFFu); ab = L; c = R; }
  else if (rule == 3) { a = (int)(cR >> 16); b = (int)(cR & 0xFFFFu); ab = R; c = L; }
  else { a = (int)(cR & 0xFFFFu); b = (int)(cR >> 16); ab = R; c = L; }
  const uint64_t *A = set_of(I, C, a), *B = set_of(I, C, b), *AB = set_of(I, C, ab), *Cc = set_of(I, C, c),
                 *D = set_of(I, C, v);
  const uint64_t* S = C.S.data();
  // Julia tcscrw on the sliced sets: tc = |out| + |x & y & ~out|
  int tcl = 0, tcr = 0, scl = 0, scr = 0, tcl1 = 0, tcr1 = 0, scl1 = 0, scr1 = 0;
  std::vector<uint64_t> ac(nw);
  for (int w = 0; w < nw; w++) {
    uint64_t nm = P.slicing ? ~S[w] : ~0ull;
    uint64_t x = (A[w] | Cc[w]) & (B[w] | D[w]);  // ref_abcacb: labels of a or c that are in b or d
    ac[w] = x;
    uint64_t ma = A[w] & nm, mb = B[w] & nm, mab = AB[w] & nm, mc = Cc[w] & nm, md = D[w] & nm, mx = x & nm;
    scl += popc(mab);
    tcl += popc(ma & mb & ~mab);
    scr += popc(md);
    tcr += popc(mab & mc & ~md);
    scl1 += popc(mx);
    tcl1 += popc(ma & mc & ~mx);
    scr1 += popc(md);
    tcr1 += popc(mx & mb & ~md);
  }
  tcl += scl, tcr += scr, tcl1 += scl1, tcr1 += scr1;
  float tc0 = lse_i(tcl, tcr), tc1 = lse_i(tcl1, tcr1);
  if (P.mode != 0) {  // cpu_ref.h:69-72: the four contractions (a,b)->ab, (ab,c)->d, (a,c)->ac, (ac,b)->d
    int c[4][4] = {};
    for (int w = 0; w < nw; w++) {
      uint64_t nm = P.slicing ? ~S[w] : ~0ull;
      uint64_t ma = A[w] & nm, mb = B[w] & nm, mab = AB[w] & nm, mc = Cc[w] & nm, md = D[w] & nm, mx = ac[w] & nm;
      count3(ma, mb, mab, c[0][0], c[0][1], c[0][2], c[0][3]);
      count3(mab, mc, md, c[1][0], c[1][1], c[1][2], c[1][3]);
      count3(ma, mc, mx, c[2][0], c[2][1], c[2][2], c[2][3]);
      count3(mx, mb, md, c[3][0], c[3][1], c[3][2], c[3][3]);
    }
    auto cost = [&](int k) { return model_cost(P, c[k][0], c[k][1], c[k][2], c[k][3]); };
    tc0 = lse_f(cost(0), cost(1));
    tc1 = lse_f(cost(2), cost(3));
  }
  int sc0 = std::max(scl, scr), sc1 = std::max(scl1, scr1);
  volatile float dtc = tc1 - tc0;
  int dsc = sc1 - sc0;
  int sc = sc0;  // Julia _sc: max(|labels(v)|, |labels(pivot)|)
  float w = ((float)std::max(sc, sc + dsc) > P.sc_target) ? P.sc_weight : 0.0f;
  volatile float wd = w * (float)dsc;
  volatile float dE = wd + dtc;
  nprop++;
  if (metropolis(rnd.b, beta, dE)) {  // Julia update_tree!, cpu_ref.h:115-121
    nacc++;
    uint32_t& cv = C.ch[v - m];
    uint32_t& cp = C.ch[ab - m];
    int l = (int)(cv & 0xFFFFu), r = (int)(cv >> 16);
    int pl = (int)(cp & 0xFFFFu), pr = (int)(cp >> 16);
    if (rule == 1) { pr = c; r = b; }        // (a,b),c -> (a,c),b
    else if (rule == 2) { pl = c; r = b; }   // (b,a),c -> (c,a),b
    else if (rule == 3) { l = b; pl = c; }   // c,(b,a) -> b,(c,a)
    else { l = b; pr = c; }                  // c,(a,b) -> b,(a,c)
    cv = (uint32_t)l | ((uint32_t)r << 16);
    cp = (uint32_t)pl | ((uint32_t)pr << 16);
    memcpy(&C.lab[(size_t)(ab - m) * nw], ac.data(), nw * 8);
  }
  return true;
}

// pre-order sweep: cpu_ref.h:89-126 (recursion into the children after the move at v)
void preorder_sweep(const Inst& I, const Par& P, Chain& C, float beta, uint32_t sweep, uint32_t chain,
                    long long& np, long long& na) {
  const int m = I.m;
  std::vector<int> st{2 * m - 2};
  while (!st.empty()) {
    int v = st.back();
    st.pop_back();
    if (v < m) continue;
    uint32_t cw = C.ch[v - m];
    if ((int)(cw & 0xFFFFu) < m && (int)(cw >> 16) < m) continue;  // empty rule set: no recursion
    visit(I, P, C, v, beta, sweep, chain, np, na);
    cw = C.ch[v - m];
    st.push_back((int)(cw >> 16));
    st.push_back((int)(cw & 0xFFFFu));
  }
}

// par sweep: cpu_ref.h:133-182.  par_band: priorities from the depth at the start of the sweep
// (cpu_ref.h:140-151); par_follow: an accepted first visit re-arms its pivot child if the sweep already
// visited it, and a follow-up visit (even priority) draws Philox with the sweep's top bit set
// (cpu_ref.h:168-175).
void par_sweep(const Inst& I, const Par& P, Chain& C, float beta, uint32_t sweep, uint32_t chain, long long& np,
               long long& na, long long* nphase) {
  const int m = I.m, n = 2 * m - 1;
  std::vector<int> parent(n, -1);
  for (int v = m; v < n; v++) {
    parent[C.ch[v - m] & 0xFFFFu] = v;
    parent[C.ch[v - m] >> 16] = v;
  }
  std::vector<uint32_t> pri(n, 0);
  for (int v = m; v < n; v++) pri[v] = par_pri((uint32_t)v, sweep, chain, P.key0);
  if (P.par_band > 0) {
    std::vector<int> dep(n, 0), st{n - 1};
    while (!st.empty()) {
      int v = st.back();
      st.pop_back();
      if (v < m) continue;
      int l = (int)(C.ch[v - m] & 0xFFFFu), r = (int)(C.ch[v - m] >> 16);
      dep[l] = dep[r] = dep[v] + 1;
      st.push_back(l);
      st.push_back(r);
    }
    for (int v = m; v < n; v++) pri[v] = par_band_pri((uint32_t)v, sweep, chain, P.key0, dep[v], P.par_band);
  }
  const uint32_t hs = mix32(sweep * 0x85EBCA77u + mix32(chain ^ P.key0));
  auto key = [&](int u) { return (pri[u] << 16) | (uint32_t)u; };
  std::vector<int> act;
  for (;;) {
    act.clear();
    for (int v = m; v < n; v++) {
      if (!pri[v]) continue;
      uint32_t kv = key(v);
      int p = parent[v];
      if (p >= 0 && pri[p] && key(p) > kv) continue;
      int l = (int)(C.ch[v - m] & 0xFFFFu), r = (int)(C.ch[v - m] >> 16);
      if (l >= m && pri[l] && key(l) > kv) continue;
      if (r >= m && pri[r] && key(r) > kv) continue;
      act.push_back(v);
    }
    if (act.empty()) break;
    if (nphase) (*nphase)++;
    for (int v : act) {
      const bool rev = (pri[v] & 1u) == 0;
      const uint32_t before = C.ch[v - m];
      visit(I, P, C, v, beta, rev ? (sweep | 0x80000000u) : sweep, chain, np, na);
      if (P.par_follow && !rev && C.ch[v - m] != before) {
        const int l0 = (int)(before & 0xFFFFu), r0 = (int)(before >> 16);
        const int Pn = (int)(C.ch[v - m] & 0xFFFFu) == l0 ? l0 : r0;  // the pivot keeps its slot
        if (!pri[Pn]) pri[Pn] = par_follow_pri((uint32_t)Pn, hs);
      }
      int l = (int)(C.ch[v - m] & 0xFFFFu), r = (int)(C.ch[v - m] >> 16);
      parent[l] = v;
      parent[r] = v;
      for (int u : {l, r})
        if (u >= m) {
          parent[C.ch[u - m] & 0xFFFFu] = u;
          parent[C.ch[u - m] >> 16] = u;
        }
      pri[v] = 0;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Whole-chain energy, float, in the lane order of the reference's warp reduction
// (eval_chain, csrc/treesa_gpu.cu:386-434): node i is accumulated by lane i % 32, then a xor
// butterfly over 16, 8, 4, 2, 1.  Glibc log2f/exp2f stand in for the device's.
// ---------------------------------------------------------------------------------------------
struct Eval {
  float lcost;
  int sc, sc_int, ncand, ns;
};
Eval eval_chain(const Inst& I, const Par& P, const Chain& C) {
  const int m = I.m, nw = I.nw;
  float acc[32];
  int scl[32], cntl[32];
  for (int l = 0; l < 32; l++) acc[l] = -INFINITY, scl[l] = 0, cntl[l] = 0;
  const uint64_t* S = P.slicing ? C.S.data() : nullptr;
  for (int i = 0; i < P.nint; i++) {
    int lane = i & 31;
    uint32_t cw = C.ch[i];
    const uint64_t *x = set_of(I, C, (int)(cw & 0xFFFFu)), *y = set_of(I, C, (int)(cw >> 16));
    const uint64_t* z = &C.lab[(size_t)i * nw];
    int Bc = 0, Mc = 0, Nc = 0, K = 0, Z = 0;
    for (int w = 0; w < nw; w++) {
      uint64_t nm = S ? ~S[w] : ~0ull;
      uint64_t zz = z[w] & nm;
      count3(x[w] & nm, y[w] & nm, zz, Bc, Mc, Nc, K);
      Z += popc(zz);
    }
    acc[lane] = lse_f(acc[lane], P.mode == 0 ? (float)(Z + K) : model_cost(P, Bc, Mc, Nc, K));
    if (Z > scl[lane]) scl[lane] = Z, cntl[lane] = 1;
    else if (Z == scl[lane]) cntl[lane]++;
  }
  for (int o = 16; o > 0; o >>= 1) {
    float nx[32];
    for (int l = 0; l < 32; l++) nx[l] = lse_f(acc[l], acc[l ^ o]);
    memcpy(acc, nx, sizeof acc);
  }
  int scmax = 0;
  for (int l = 0; l < 32; l++) scmax = std::max(scmax, scl[l]);
  int cnt = 0, ns = 0;
  for (int l = 0; l < 32; l++) cnt += scl[l] == scmax ? cntl[l] : 0;
  if (S)
    for (int w = 0; w < nw; w++) ns += popc(S[w]);
  int sc = std::max(scmax, P.leaf_sc);
  if (S && P.leaf_sc > scmax) {
    int ll = 0;
    for (int i = 0; i < m; i++) {
      int Z = 0;
      for (int w = 0; w < nw; w++) Z += popc(I.leaf[(size_t)i * nw + w] & ~S[w]);
      ll = std::max(ll, Z);
    }
    sc = std::max(scmax, ll);
  }
  return Eval{acc[0], sc, scmax, cnt, ns};
}

float slice_energy(const Eval& e, const Par& P) {  // treesa_gpu.cu:436-439
  volatile float pen = (float)e.sc > P.sc_target ? P.sc_weight * ((float)e.sc - P.sc_target) : 0.0f;
  volatile float a = (float)e.ns + e.lcost;
  volatile float r = a + pen;
  return r;
}

int nth_set(const uint64_t* A, const uint64_t* S, int nw, int n) {  // nth_label, treesa_gpu.cu:124-133
  for (int w = 0; w < nw; w++) {
    uint64_t a = A[w] & (S ? ~S[w] : ~0ull);
    int c = popc(a);
    if (n < c) {
      for (int k = 0; k < n; k++) a &= a - 1;
      return w * 64 + __builtin_ctzll(a);
    }
    n -= c;
  }
  return -1;
}

// slice moves after a sweep: slice_step, treesa_gpu.cu:445-502
void slice_step(const Inst& I, const Par& P, Chain& C, float beta, uint32_t sweep, uint32_t chain, long long& nsp,
                long long& nsa) {
  const int nw = I.nw;
  Eval cur = eval_chain(I, P, C);
  float Ecur = slice_energy(cur, P);
  uint64_t* S = C.S.data();
  for (int j = 0; j < P.slice_moves; j++) {
    R4 r1 = philox(0x10000u + 2u * j, sweep, chain, 0u, P.key0, P.key1);
    R4 r2 = philox(0x10001u + 2u * j, sweep, chain, 0u, P.key0, P.key1);
    int type;
    if (cur.ns == 0) type = 0;
    else if (cur.ns >= P.max_slices) type = (r1.a >> 31) ? 1 : 2;
    else type = r1.a < 0x80000000u ? 0 : (r1.a < 0xC0000000u ? 1 : 2);
    int ladd = -1, lrem = -1;
    if (type != 1 && cur.ncand > 0 && cur.sc_int > 0) {
      int rr = (int)(r1.b % (uint32_t)cur.ncand), node = -1;
      for (int i = 0; i < P.nint; i++) {
        int Z = 0;
        for (int w = 0; w < nw; w++) Z += popc(C.lab[(size_t)i * nw + w] & ~S[w]);
        if (Z == cur.sc_int) {
          if (rr == 0) {
            node = i;
            break;
          }
          rr--;
        }
      }
      if (node >= 0) ladd = nth_set(&C.lab[(size_t)node * nw], S, nw, (int)(r1.c % (uint32_t)cur.sc_int));
    }
    if (type != 0) lrem = nth_set(S, nullptr, nw, (int)(r1.d % (uint32_t)cur.ns));
    if (type == 2 && ladd < 0) type = 1;
    if (type == 0 && ladd < 0) continue;
    if (type != 1) S[ladd >> 6] |= 1ull << (ladd & 63);
    if (type != 0) S[lrem >> 6] &= ~(1ull << (lrem & 63));
    Eval nxt = eval_chain(I, P, C);
    float Enew = slice_energy(nxt, P);
    nsp++;
    volatile float dE = Enew - Ecur;
    if (metropolis(r2.a, beta, dE)) {
      nsa++;
      cur = nxt;
      Ecur = Enew;
    } else {
      if (type != 1) S[ladd >> 6] &= ~(1ull << (ladd & 63));
      if (type != 0) S[lrem >> 6] |= 1ull << (lrem & 63);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host double-precision energies and the slicer repair (treesa_gpu.cu:1182-1274)
// ---------------------------------------------------------------------------------------------
double gpu_time_d(int B, int M_, int N, int K, const Models& M) {  // treesa_gpu.cu:1182-1186
  double ops = exp2((double)(1 + B + std::max(M_, M.m0) + std::max(N, M.n0) + std::max(K, M.k0)));
  double bits = exp2((double)(B + M_ + K)) + exp2((double)(B + N + K)) + exp2((double)(B + M_ + N));
  return std::max(ops / exp2((double)M.lpeak), bits / exp2((double)M.lbw)) + exp2((double)M.llaunch);
}
double h100_time_d(int B, int M_, int N, int K, const Models& M) {  // treesa_gpu.cu:1189-1203
  auto e = [](float l) { return exp2((double)l); };
  if (B + M_ + N <= M.small_rank) return e(M.lsmall_cell) * exp2((double)(B + M_ + N + K));
  double a = exp2((double)(B + M_ + K)), b = exp2((double)(B + N + K)), c = exp2((double)(B + M_ + N));
  double moved = a + b + c;
  double perm = e(M.lperm2) * (a + b);
  double best = e(M.lcc_bit) * moved + e(M.lcc_cell) * exp2((double)(B + M_ + N + K));
  if (K >= 7 && std::max(M_, N) >= 5) {
    double tc = e(M.ltc_bit) * moved + e(M.ltc_pad) * exp2((double)(B + std::max(M_, 6) + std::max(N, 6) + std::max(K, 8))) +
                e(M.ltc_out) * c;
    best = std::min(best, tc);
  }
  return e(M.l3launch) + perm + best;
}

struct HostE {
  double tc = 0, time = 0, time2 = 0;
  int sc = 0, ns = 0;
};
HostE host_energy(const Inst& I, const Models& Mo, const uint64_t* lab, const uint32_t* ch, const uint64_t* S) {
  const int nw = I.nw, m = I.m;  // treesa_gpu.cu:1206-1244
  HostE E;
  std::vector<uint64_t> nm(nw, ~0ull);
  if (S)
    for (int w = 0; w < nw; w++) nm[w] = ~S[w], E.ns += popc(S[w]);
  for (int i = 0; i < m; i++) {
    int z = 0;
    for (int w = 0; w < nw; w++) z += popc(I.leaf[(size_t)i * nw + w] & nm[w]);
    E.sc = std::max(E.sc, z);
  }
  double mx = -1e300;
  std::vector<double> tcs;
  for (int i = 0; i < m - 1; i++) {
    int l = (int)(ch[i] & 0xFFFFu), r = (int)(ch[i] >> 16);
    const uint64_t* x = l >= m ? lab + (size_t)(l - m) * nw : &I.leaf[(size_t)l * nw];
    const uint64_t* y = r >= m ? lab + (size_t)(r - m) * nw : &I.leaf[(size_t)r * nw];
    const uint64_t* z = lab + (size_t)i * nw;
    int B = 0, M_ = 0, N = 0, K = 0, sz = 0;
    for (int w = 0; w < nw; w++) {
      uint64_t a = x[w] & nm[w], b = y[w] & nm[w], c = z[w] & nm[w];
      B += popc(a & b & c);
      M_ += popc(a & ~b & c);
      N += popc(~a & b & c);
      K += popc(a & b & ~c);
      sz += popc(c);
    }
    double t = B + M_ + N + K;
    tcs.push_back(t);
    mx = std::max(mx, t);
    E.sc = std::max(E.sc, sz);
    E.time += gpu_time_d(B, M_, N, K, Mo);
    E.time2 += h100_time_d(B, M_, N, K, Mo);
  }
  double s = 0;
  for (double t : tcs) s += exp2(t - mx);
  E.tc = mx + log2(s);
  return E;
}

int greedy_repair(const Inst& I, const uint64_t* lab, uint64_t* S, double sc_target) {  // :1248-1274
  const int nw = I.nw, m = I.m;
  int added = 0;
  for (;;) {
    int scmax = 0;
    std::vector<int> sizes(2 * m - 1);
    auto so = [&](int v) -> const uint64_t* { return v < m ? &I.leaf[(size_t)v * nw] : lab + (size_t)(v - m) * nw; };
    for (int v = 0; v < 2 * m - 1; v++) {
      const uint64_t* a = so(v);
      int z = 0;
      for (int w = 0; w < nw; w++) z += popc(a[w] & ~S[w]);
      sizes[v] = z;
      scmax = std::max(scmax, z);
    }
    if (scmax <= sc_target || scmax == 0) return added;
    std::vector<int> freq(I.nlab, 0);
    for (int v = 0; v < 2 * m - 1; v++)
      if (sizes[v] == scmax) {
        const uint64_t* a = so(v);
        for (int l = 0; l < I.nlab; l++)
          if ((a[l >> 6] & ~S[l >> 6]) >> (l & 63) & 1ull) freq[l]++;
      }
    int best = (int)(std::max_element(freq.begin(), freq.end()) - freq.begin());
    S[best >> 6] |= 1ull << (best & 63);
    added++;
  }
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

Par make_par(const Inst& I, const tsa_options* O) {  // Runner ctor, treesa_gpu.cu:1435-1460
  Par P{};
  P.m = I.m;
  P.nint = I.m - 1;
  P.nw = I.nw;
  P.leaf_sc = 0;
  for (auto& ix : I.ixs) P.leaf_sc = std::max(P.leaf_sc, (int)ix.size());
  P.slicing = O->slicing ? 1 : 0;
  P.slice_moves = O->slicing ? O->slice_moves : 0;
  P.slice_every = std::max(1, O->slice_every);
  P.max_slices = O->max_slices > 0 ? O->max_slices : I.nlab;
  P.sc_target = (float)O->sc_target;
  P.sc_weight = (float)O->sc_weight;
  P.par_band = O->par_band;
  P.par_follow = O->par_follow ? 1 : 0;
  P.mode = O->mode;
  P.mo = make_models(O->gpu_model, O->h100_model);
  uint64_t k = splitmix64(O->seed);
  P.key0 = (uint32_t)k;
  P.key1 = (uint32_t)(k >> 32);
  return P;
}

bool init_chain(const Inst& I, const tsa_options* O, int c, Chain& C, const std::vector<uint64_t>& S0) {
  const int nint = I.m - 1;
  C.ch.resize(nint);
  C.lab.assign((size_t)nint * I.nw, 0);
  C.S = S0;
  if (O->ntrees > 0 && O->init_trees)
    memcpy(C.ch.data(), O->init_trees + (size_t)(c % O->ntrees) * nint, nint * 4);
  else
    C.ch = random_tree(I.m, splitmix64(O->seed * 1000003ULL + (uint64_t)c));  // treesa_gpu.cu:1608
  return labels_from_topology(I, C.ch.data(), C.lab.data());
}

}  // namespace

extern "C" {

// The whole optimize run (Runner<W>::run_anneal, csrc/treesa_gpu.cu:1756-1923), single process.
int orc_run(const tsa_instance* inst, const tsa_options* O, tsa_result* res, char* err, size_t errlen) {
  memset(res, 0, sizeof *res);
  Inst I;
  if (!load_instance(inst, I, err, errlen)) return TSA_ERR_ARG;
  if (O->nchains < 1 || O->niters < 0 || O->nbetas < 1) {
    snprintf(err, errlen, "oracle: bad nchains/niters/betas");
    return TSA_ERR_ARG;
  }
  Par P = make_par(I, O);
  const Models Mo = make_models(O->gpu_model, O->h100_model);
  const int nch = O->nchains, nint = P.nint, nw = I.nw;
  std::vector<float> betas(O->betas, O->betas + O->nbetas);
  if (O->max_levels > 0 && (int)betas.size() > O->max_levels) betas.resize(O->max_levels);
  // level schedule (treesa_gpu.cu:1758-1764): stage 2 continues the population in mode2
  std::vector<int> lmode(betas.size(), O->mode), lniters(betas.size(), O->niters);
  if (O->betas2 && O->nbetas2 > 0)
    for (int k = 0; k < O->nbetas2; k++) {
      betas.push_back(O->betas2[k]);
      lmode.push_back(O->mode2);
      lniters.push_back(O->niters2 > 0 ? O->niters2 : O->niters);
    }
  int mode = O->mode;
  std::vector<uint64_t> S0(nw, 0);
  for (int k = 0; k < O->ninit_slices; k++) {
    int l = O->init_slices[k];
    if (l < 0 || l >= I.nlab) {
      snprintf(err, errlen, "oracle: bad init slice label");
      return TSA_ERR_ARG;
    }
    S0[l >> 6] |= 1ull << (l & 63);
  }
  double t_start = now_s();
  std::vector<Chain> pop(nch);
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 4) reduction(+ : bad)
  for (int c = 0; c < nch; c++)
    if (!init_chain(I, O, c, pop[c], S0)) bad++;
  if (bad) {
    snprintf(err, errlen, "oracle: invalid initial tree");
    return TSA_ERR_ARG;
  }
  double t_init = now_s() - t_start;
  double t0 = now_s();
  auto energyE = [&](float lc, int sc, int ns) -> double {  // treesa_gpu.cu:1750-1753
    return (double)ns + (double)lc + O->sc_weight * std::max(0.0, (double)sc - O->sc_target);
  };
  auto score = [&](float lc, int sc, int ns) -> double {  // treesa_gpu.cu:1737-1747
    if (O->slicing) return (double)ns + (double)lc + 1000.0 * std::max(0.0, (double)sc - O->sc_target);
    if (O->select_sc) return 4096.0 * std::max(0.0, (double)sc - O->sc_target) + (double)lc;
    if (mode != 0) return energyE(lc, sc, ns);
    double tc = (double)lc;
    if ((double)sc <= O->sc_target || O->sc_weight <= 0) return tc;
    double pen = log2(O->sc_weight) + (double)sc + log2(1.0 - exp2(O->sc_target - (double)sc));
    double mx = std::max(tc, pen), mn = std::min(tc, pen);
    return mx + log2(1.0 + exp2(mn - mx));
  };
  double best_score = INFINITY;
  int best_chain = -1;
  Chain best;
  std::vector<int> family(nch), nfam(nch);
  std::iota(family.begin(), family.end(), 0);
  std::vector<double> trace;
  std::mt19937_64 hrng(splitmix64(O->seed + 777));
  float beta_last = betas[0];
  int nresample = 0;
  uint32_t sweep_ctr = 0;
  long long tot_np = 0, tot_na = 0, tot_nsp = 0, tot_nsa = 0, tot_ph = 0;
  std::vector<float> lc(nch);
  std::vector<int> sc(nch), ns(nch);
  const int ee = std::max(1, O->eval_every);
  for (size_t lev = 0; lev < betas.size(); lev++) {
    if (lmode[lev] != mode) {  // stage switch (treesa_gpu.cu:1793-1799): the incumbent rescored in the new energy
      HostE H1 = host_energy(I, Mo, best.lab.data(), best.ch.data(), O->slicing ? best.S.data() : nullptr);
      mode = lmode[lev];
      P.mode = mode;
      best_score = score((float)log2(mode == 1 ? H1.time : H1.time2), H1.sc, H1.ns);
      beta_last = betas[lev];
    }
    const float beta = betas[lev];
    const uint32_t sw0 = sweep_ctr;
    const int nit = lniters[lev];
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : tot_np, tot_na, tot_nsp, tot_nsa, tot_ph)
    for (int c = 0; c < nch; c++) {
      long long np = 0, na = 0, nsp = 0, nsa = 0, ph = 0;
      for (int it = 0; it < nit; it++) {
        uint32_t sw = sw0 + (uint32_t)it;
        if (O->order == TSA_ORDER_PAR) par_sweep(I, P, pop[c], beta, sw, (uint32_t)c, np, na, &ph);
        else preorder_sweep(I, P, pop[c], beta, sw, (uint32_t)c, np, na);
        if (P.slice_moves > 0 && (sw + 1) % (uint32_t)P.slice_every == 0)
          slice_step(I, P, pop[c], beta, sw, (uint32_t)c, nsp, nsa);
      }
      tot_np += np, tot_na += na, tot_nsp += nsp, tot_nsa += nsa, tot_ph += ph;
    }
    sweep_ctr += (uint32_t)nit;
    bool last = lev + 1 == betas.size();
    bool switching = !last && lmode[lev + 1] != mode;  // no population step across an energy change
    if ((int)(lev % ee) == ee - 1 || last || switching) {
#pragma omp parallel for schedule(dynamic, 4)
      for (int c = 0; c < nch; c++) {
        Eval e = eval_chain(I, P, pop[c]);
        lc[c] = e.lcost, sc[c] = e.sc, ns[c] = e.ns;
      }
      int bi = 0;
      double bs = INFINITY, meanE = 0, meanNs = 0;
      for (int c = 0; c < nch; c++) {
        double s = score(lc[c], sc[c], ns[c]);
        if (s < bs) bs = s, bi = c;
        meanE += energyE(lc[c], sc[c], ns[c]);
        meanNs += ns[c];
      }
      meanE /= nch;
      meanNs /= nch;
      if (bs < best_score) {
        best_score = bs;
        best_chain = bi;
        best = pop[bi];
      }
      std::fill(nfam.begin(), nfam.end(), 0);
      int nf = 0;
      for (int c = 0; c < nch; c++)
        if (nfam[family[c]]++ == 0) nf++;
      double row[10] = {now_s() - t0, (double)lev, (double)betas[lev], (double)lc[bi], (double)sc[bi], meanE,
                        (double)nf, (double)mode, (double)ns[bi], meanNs};
      trace.insert(trace.end(), row, row + 10);
      std::vector<int> anc;
      if (!last && !switching && O->scheme == TSA_SCHEME_PA) {  // treesa_gpu.cu:1837-1856
        double db = betas[lev + 1] - beta_last;
        beta_last = betas[lev + 1];
        std::vector<double> w(nch);
        double Emin = INFINITY;
        for (int c = 0; c < nch; c++) Emin = std::min(Emin, energyE(lc[c], sc[c], ns[c]));
        double wsum = 0;
        for (int c = 0; c < nch; c++) {
          w[c] = exp(-db * (energyE(lc[c], sc[c], ns[c]) - Emin));
          wsum += w[c];
        }
        anc.assign(nch, 0);
        double u = std::uniform_real_distribution<double>(0, 1)(hrng), acc = 0;
        int j = 0;
        for (int c = 0; c < nch; c++) {
          acc += w[c] / wsum * nch;
          while (j < nch && j + u < acc) anc[j++] = c;
        }
        while (j < nch) anc[j++] = nch - 1;
      } else if (!last && !switching && O->scheme == TSA_SCHEME_TRUNC) {  // treesa_gpu.cu:1857-1869
        std::vector<int> idx(nch);
        std::iota(idx.begin(), idx.end(), 0);
        std::sort(idx.begin(), idx.end(),
                  [&](int a, int b) { return energyE(lc[a], sc[a], ns[a]) < energyE(lc[b], sc[b], ns[b]); });
        anc.resize(nch);
        std::iota(anc.begin(), anc.end(), 0);
        int nrep = (int)(O->trunc_frac * nch);
        for (int k = 0; k < nrep; k++) anc[idx[nch - 1 - k]] = idx[k];
      }
      if (!anc.empty()) {  // resample, treesa_gpu.cu:1925-1933
        std::vector<Chain> np2(nch);
        std::vector<int> nfm(nch);
        for (int c = 0; c < nch; c++) np2[c] = pop[anc[c]], nfm[c] = family[anc[c]];
        pop.swap(np2);
        family.swap(nfm);
        nresample++;
      }
    }
  }
  double t_anneal = now_s() - t0;
  // finalize, treesa_gpu.cu:1878-1919
  if (best_chain < 0) {
    snprintf(err, errlen, "oracle: no level evaluated");
    return TSA_ERR_ARG;
  }
  std::vector<uint64_t> lab2((size_t)nint * nw);
  bool valid = labels_from_topology(I, best.ch.data(), lab2.data());
  bool labels_ok = valid && lab2 == best.lab;
  int n_repair = 0;
  if (O->slicing && valid) n_repair = greedy_repair(I, lab2.data(), best.S.data(), O->sc_target);
  HostE HE = host_energy(I, Mo, lab2.data(), best.ch.data(), O->slicing ? best.S.data() : nullptr);
  res->m = I.m;
  res->tree = (uint32_t*)malloc(sizeof(uint32_t) * nint);
  memcpy(res->tree, best.ch.data(), nint * 4);
  std::vector<int> sl;
  if (O->slicing)
    for (int l = 0; l < I.nlab; l++)
      if (best.S[l >> 6] >> (l & 63) & 1ull) sl.push_back(l);
  res->nsliced = (int)sl.size();
  res->sliced = (int32_t*)malloc(sizeof(int32_t) * std::max<size_t>(1, sl.size()));
  if (!sl.empty()) memcpy(res->sliced, sl.data(), sl.size() * 4);
  res->tc = HE.tc;
  res->sc = HE.sc;
  res->gpu_time = HE.time;
  res->h100_time = HE.time2;
  res->valid = valid;
  res->labels_ok = labels_ok;
  res->best_chain = best_chain;
  res->slicing = O->slicing ? 1 : 0;
  res->n_repair = n_repair;
  res->tc_total = HE.tc + HE.ns;
  res->gpu_time_total = HE.time * exp2((double)HE.ns);
  res->h100_time_total = HE.time2 * exp2((double)HE.ns);
  res->t_anneal = t_anneal;
  res->t_init = t_init;
  res->kernel_s = t_anneal;
  res->proposals = (uint64_t)tot_np;
  res->accepts = (uint64_t)tot_na;
  res->warp_steps = (uint64_t)tot_ph;
  res->node_visits = (uint64_t)sweep_ctr * (uint64_t)nch * (uint64_t)nint;
  res->slice_proposals = (uint64_t)tot_nsp;
  res->slice_accepts = (uint64_t)tot_nsa;
  res->nchains = nch;
  res->niters = O->niters;
  res->nlevels = (int)betas.size();
  res->total_sweeps = (int)sweep_ctr;
  res->W = 0;
  res->nw = nw;
  res->scheme = O->scheme;
  res->mode = O->mode;
  res->nresample = nresample;
  res->order = O->order;
  res->ntrace = (int)(trace.size() / 10);
  res->trace = (double*)malloc(sizeof(double) * std::max<size_t>(1, trace.size()));
  if (!trace.empty()) memcpy(res->trace, trace.data(), trace.size() * 8);
  snprintf(res->kernel, sizeof res->kernel, "oracle");
  return valid && labels_ok ? TSA_OK : TSA_ERR_INVALID;
}

void orc_result_free(tsa_result* r) {
  free(r->tree);
  free(r->sliced);
  free(r->trace);
  r->tree = nullptr;
  r->sliced = nullptr;
  r->trace = nullptr;
}

// Trajectory oracle (the --check [4] comparison, csrc/treesa_gpu.cu:2012-2052): chains c0..c0+nch-1
// start from trees_in (and slice sets S_in, [nch][nw] u64, or NULL) and run nbetas levels of niters
// sweeps with sweep id lev*niters+it; fixed slice sets (no slice moves).  Writes the final trees and
// labels.  counters: [0] proposals, [1] accepts, [2] phases.
int orc_sweeps(const tsa_instance* inst, int order, int par_band, int par_follow, int mode, uint64_t seed,
               double sc_target,
               double sc_weight, const float* betas, int nbetas, int niters, int nch, int c0,
               const uint32_t* trees_in, const uint64_t* S_in, uint32_t* trees_out, uint64_t* labels_out,
               long long* counters, char* err, size_t errlen) {
  Inst I;
  if (!load_instance(inst, I, err, errlen)) return TSA_ERR_ARG;
  tsa_options O{};
  O.par_band = par_band;
  O.par_follow = par_follow;
  O.mode = mode;
  O.sc_target = sc_target;
  O.sc_weight = sc_weight;
  O.seed = seed;
  O.slicing = S_in != nullptr;
  O.slice_every = 1;
  Par P = make_par(I, &O);
  P.slice_moves = 0;
  const int nint = I.m - 1, nw = I.nw;
  long long np = 0, na = 0, ph = 0;
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : np, na, ph, bad)
  for (int k = 0; k < nch; k++) {
    Chain C;
    C.ch.assign(trees_in + (size_t)k * nint, trees_in + (size_t)(k + 1) * nint);
    C.lab.assign((size_t)nint * nw, 0);
    C.S.assign(nw, 0);
    if (S_in) memcpy(C.S.data(), S_in + (size_t)k * nw, nw * 8);
    if (!labels_from_topology(I, C.ch.data(), C.lab.data())) {
      bad++;
      continue;
    }
    long long a = 0, b = 0, p = 0;
    for (int lev = 0; lev < nbetas; lev++)
      for (int it = 0; it < niters; it++) {
        uint32_t sw = (uint32_t)(lev * niters + it);
        if (order == TSA_ORDER_PAR) par_sweep(I, P, C, betas[lev], sw, (uint32_t)(c0 + k), a, b, &p);
        else preorder_sweep(I, P, C, betas[lev], sw, (uint32_t)(c0 + k), a, b);
      }
    np += a, na += b, ph += p;
    memcpy(trees_out + (size_t)k * nint, C.ch.data(), nint * 4);
    if (labels_out) memcpy(labels_out + (size_t)k * nint * nw, C.lab.data(), (size_t)nint * nw * 8);
  }
  if (counters) counters[0] = np, counters[1] = na, counters[2] = ph;
  if (bad) {
    snprintf(err, errlen, "oracle: invalid tree");
    return TSA_ERR_ARG;
  }
  return TSA_OK;
}

// Host-init helpers for tests: the random start tree of global chain c and topology labels.
void orc_random_tree(int m, uint64_t seed, int chain, uint32_t* out) {
  std::vector<uint32_t> t = random_tree(m, splitmix64(seed * 1000003ULL + (uint64_t)chain));
  memcpy(out, t.data(), (m - 1) * 4);
}
int orc_labels(const tsa_instance* inst, const uint32_t* tree, uint64_t* labels, char* err, size_t errlen) {
  Inst I;
  if (!load_instance(inst, I, err, errlen)) return TSA_ERR_ARG;
  return labels_from_topology(I, tree, labels) ? TSA_OK : TSA_ERR_INVALID;
}
// Float per-chain energy of one tree (eval_chain semantics) and host double tc/sc.
int orc_energy(const tsa_instance* inst, const uint32_t* tree, const uint64_t* S, float* lcost, int* sc, int* ns,
               double* tc_host, int* sc_host, char* err, size_t errlen) {
  Inst I;
  if (!load_instance(inst, I, err, errlen)) return TSA_ERR_ARG;
  tsa_options O{};
  O.slicing = S != nullptr;
  O.sc_target = 1e9;
  Par P = make_par(I, &O);
  Chain C;
  C.ch.assign(tree, tree + I.m - 1);
  C.lab.assign((size_t)(I.m - 1) * I.nw, 0);
  C.S.assign(I.nw, 0);
  if (S) memcpy(C.S.data(), S, I.nw * 8);
  if (!labels_from_topology(I, C.ch.data(), C.lab.data())) return TSA_ERR_INVALID;
  Eval e = eval_chain(I, P, C);
  *lcost = e.lcost, *sc = e.sc, *ns = e.ns;
  HostE H = host_energy(I, make_models(nullptr, nullptr), C.lab.data(), C.ch.data(), S);
  *tc_host = H.tc, *sc_host = H.sc;
  return TSA_OK;
}

// Checksum of the host libm's expf over the float bit patterns [lo, hi] (same formula as the
// product's tsa_expf_selftest).
uint64_t orc_expf_checksum(uint32_t lo, uint32_t hi) {
  uint64_t acc = 0;
  const long long n = (long long)hi - (long long)lo + 1;
#pragma omp parallel for reduction(+ : acc) schedule(static)
  for (long long k = 0; k < n; k++) {
    uint32_t xb = lo + (uint32_t)k;
    float x;
    memcpy(&x, &xb, 4);
    float g = expf(x);
    uint32_t gb;
    memcpy(&gb, &g, 4);
    acc += (uint64_t)(gb ^ (xb * 0x9E3779B1u));
  }
  return acc;
}

}  // extern "C"
