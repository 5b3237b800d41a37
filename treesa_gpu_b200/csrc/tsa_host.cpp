// tsa_host.cpp -- host side of libtreesa_b200.so: the C ABI (include/treesa_b200.h), chain
// initialization, the beta-level scheduler with best-of-N / population annealing / truncation selection,
// and the finalize step.  Follows the reference's Runner<W> (csrc/treesa_gpu.cu:1416-1933) in
// semantics; all state lives in a session object (no global mutable state), so concurrent calls on
// different devices are independent.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <omp.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <functional>
#include <map>
#include <mutex>
#include <numeric>
#include <random>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/treesa_b200.h"
#include "tsa_comm.h"
#include "tsa_core.h"
#include "tsa_exp_table.h"
#include "tsa_kernels.cuh"

using tsa::Layout;

namespace {

void set_err(char* err, size_t n, const char* fmt, ...) {
  if (!err || n == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, n, fmt, ap);
  va_end(ap);
}

#define CKR(x)                                                                                 \
  do {                                                                                         \
    cudaError_t e_ = (x);                                                                      \
    if (e_ != cudaSuccess) {                                                                   \
      set_err(err, errlen, "CUDA error %s at %s:%d", cudaGetErrorString(e_), __FILE__, __LINE__); \
      return TSA_ERR_CUDA;                                                                     \
    }                                                                                          \
  } while (0)

// Process-wide cache of device and pinned host blocks.  One-shot tsa_run calls of one workload reuse the
// previous call's buffers instead of paying cudaMalloc / cudaMallocHost and the synchronizing frees on
// every call.  A freed block is kept for a later request of the same (device, kind, size) while the
// cache holds at most kPoolCap[kind] bytes; tsa_release_cached_memory() empties it.  Blocks go back to
// the cache only after the session's streams are idle.
struct BlockPool {
  static constexpr size_t kPoolCap[2] = {size_t(8) << 30, size_t(1) << 30};  // device, pinned host
  struct Key {
    int device, kind;
    size_t bytes;
    bool operator<(const Key& o) const { return std::tie(device, kind, bytes) < std::tie(o.device, o.kind, o.bytes); }
  };
  std::mutex mu;
  std::multimap<Key, void*> idle;
  std::map<void*, Key> live;
  size_t held[2] = {0, 0};
};
BlockPool& block_pool() {
  static BlockPool* P = new BlockPool();  // never destroyed: blocks may outlive static destruction order
  return *P;
}
void raw_free(int kind, void* p) {
  if (kind == 0)
    cudaFree(p);
  else
    cudaFreeHost(p);
}
// kind 0: device memory of the current device; 1: pinned host memory
cudaError_t pool_alloc(int kind, void** out, size_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  bytes = std::max<size_t>(bytes, 1);
  BlockPool& P = block_pool();
  const BlockPool::Key k{kind == 0 ? dev : -1, kind, bytes};
  {
    std::lock_guard<std::mutex> g(P.mu);
    auto it = P.idle.find(k);
    if (it != P.idle.end()) {
      *out = it->second;
      P.idle.erase(it);
      P.held[kind] -= bytes;
      P.live[*out] = k;
      return cudaSuccess;
    }
  }
  e = kind == 0 ? cudaMalloc(out, bytes) : cudaMallocHost(out, bytes);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(P.mu);
  P.live[*out] = k;
  return cudaSuccess;
}
template <typename T>
cudaError_t pool_alloc(int kind, T** out, size_t bytes) {
  return pool_alloc(kind, reinterpret_cast<void**>(out), bytes);
}
void pool_free(void* p) {
  if (!p) return;
  BlockPool& P = block_pool();
  std::lock_guard<std::mutex> g(P.mu);
  auto it = P.live.find(p);
  if (it == P.live.end()) return;
  const BlockPool::Key k = it->second;
  P.live.erase(it);
  if (P.held[k.kind] + k.bytes <= BlockPool::kPoolCap[k.kind]) {
    P.idle.emplace(k, p);
    P.held[k.kind] += k.bytes;
  } else {
    raw_free(k.kind, p);
  }
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

uint64_t splitmix64(uint64_t x) {  // csrc/treesa_gpu.cu:1408-1413
  x += 0x9E3779B97F4A7C15ULL;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
  return x ^ (x >> 31);
}

inline uint32_t rup(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }
inline int popc(uint64_t x) { return __builtin_popcountll(x); }

// ------------------------------------------------------------------------------------------------
// Instance (read_instance semantics, csrc/treesa_gpu.cu:1035-1073)
// ------------------------------------------------------------------------------------------------
struct Inst {
  int m = 0, nlab = 0, nw = 1;
  std::vector<std::vector<int>> ixs;
  std::vector<int> iy, total;
  std::vector<char> in_iy;
  std::vector<uint64_t> leaf;  // [m][nw]
  int leaf_sc = 0;
};

int load_inst(const tsa_instance* I, Inst& S, char* err, size_t errlen) {
  if (!I || !I->ix_offsets || (I->m > 0 && !I->ix_labels)) {
    set_err(err, errlen, "null instance");
    return TSA_ERR_ARG;
  }
  if (I->m < 3) {
    set_err(err, errlen, "need at least 3 tensors");
    return TSA_ERR_ARG;
  }
  if (2 * (long long)I->m - 1 > 65535) {
    set_err(err, errlen, "too many tensors (node ids are 16-bit)");
    return TSA_ERR_ARG;
  }
  if (I->nlab < 0 || I->nlab > 32767) {
    set_err(err, errlen, "label count out of range");
    return TSA_ERR_ARG;
  }
  S.m = I->m;
  S.nlab = I->nlab;
  int nw = (I->nlab + 63) / 64;
  if (nw < 1) nw = 1;
  if (nw > 1 && (nw & 1)) nw++;  // 16-byte aligned label sets
  S.nw = nw;
  S.ixs.assign(S.m, {});
  S.total.assign(S.nlab, 0);
  S.in_iy.assign(S.nlab, 0);
  for (int i = 0; i < S.m; i++) {
    int a = I->ix_offsets[i], b = I->ix_offsets[i + 1];
    if (b < a) {
      set_err(err, errlen, "bad ix offsets");
      return TSA_ERR_ARG;
    }
    S.ixs[i].assign(I->ix_labels + a, I->ix_labels + b);
    std::sort(S.ixs[i].begin(), S.ixs[i].end());
    if (std::adjacent_find(S.ixs[i].begin(), S.ixs[i].end()) != S.ixs[i].end()) {
      set_err(err, errlen, "repeated label inside one tensor is not supported");
      return TSA_ERR_ARG;
    }
    for (int l : S.ixs[i]) {
      if (l < 0 || l >= S.nlab) {
        set_err(err, errlen, "label out of range");
        return TSA_ERR_ARG;
      }
      S.total[l]++;
    }
    S.leaf_sc = std::max(S.leaf_sc, (int)S.ixs[i].size());
  }
  for (int j = 0; j < I->niy; j++) {
    int l = I->iy[j];
    if (l < 0 || l >= S.nlab) {
      set_err(err, errlen, "open label out of range");
      return TSA_ERR_ARG;
    }
    S.iy.push_back(l);
    S.in_iy[l] = 1;
  }
  S.leaf.assign((size_t)S.m * nw, 0);
  for (int i = 0; i < S.m; i++)
    for (int l : S.ixs[i]) S.leaf[(size_t)i * nw + (l >> 6)] |= 1ull << (l & 63);
  return TSA_OK;
}

// ------------------------------------------------------------------------------------------------
// Trees and labels
// ------------------------------------------------------------------------------------------------
// Julia random_exprtree as in csrc/treesa_gpu.cu:1101-1123 (same std::mt19937_64 draws)
std::vector<uint32_t> random_tree(int m, uint64_t seed) {
  std::mt19937_64 rng(seed);
  std::vector<uint32_t> ch(m - 1);
  int next = m;
  std::function<int(const std::vector<int>&)> build = [&](const std::vector<int>& xs) -> int {
    const int n = (int)xs.size();
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
    a.reserve(n);
    b.reserve(n);
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

// Output labels of every internal node from the topology (the rule of labels_from_topology,
// csrc/treesa_gpu.cu:1149-1172: l is an output of v iff it occurs in v's subtree and also outside it,
// or is open).  Computed by closure: z(v) = (z(left) | z(right)) minus the labels that close at v,
// i.e. whose occurrences all lie in v's subtree for the first time (the LCA of the occurrences, or the
// parent of the only occurrence); open labels never close.  O(m * nw + sum of occurrences * depth).
// Returns false if ch is not a binary tree over all 2m-1 nodes rooted at 2m-2.
bool topo_labels(const Inst& I, const uint32_t* ch, uint64_t* lab) {
  const int m = I.m, n = 2 * m - 1, nw = I.nw;
  std::vector<int> parent(n, -1), depth(n, 0), order;
  order.reserve(m - 1);
  {
    std::vector<char> seen(n, 0);
    std::vector<int> st{n - 1};
    int nseen = 0;
    while (!st.empty()) {
      int v = st.back();
      st.pop_back();
      if (v < 0 || v >= n || seen[v]) return false;
      seen[v] = 1;
      nseen++;
      if (v >= m) {
        order.push_back(v);
        int l = (int)(ch[v - m] & 0xFFFFu), r = (int)(ch[v - m] >> 16);
        for (int u : {l, r}) {
          if (u < 0 || u >= n) return false;
          if (!seen[u]) {
            parent[u] = v;
            depth[u] = depth[v] + 1;
          }
          st.push_back(u);
        }
      }
    }
    if (nseen != n) return false;
  }
  // closing node of every non-open label
  std::vector<std::vector<int>> closes(m - 1);
  std::vector<int> first(I.nlab, -1), lca(I.nlab, -1);
  for (int t = 0; t < m; t++)
    for (int l : I.ixs[t]) {
      if (I.in_iy[l]) continue;
      if (lca[l] < 0) {
        lca[l] = t;
        continue;
      }
      int a = lca[l], b = t;
      while (depth[a] > depth[b]) a = parent[a];
      while (depth[b] > depth[a]) b = parent[b];
      while (a != b) a = parent[a], b = parent[b];
      lca[l] = a;
    }
  for (int l = 0; l < I.nlab; l++) {
    if (lca[l] < 0) continue;
    int v = lca[l] < m ? parent[lca[l]] : lca[l];  // a single occurrence closes at its parent
    closes[v - m].push_back(l);
  }
  for (int k = (int)order.size() - 1; k >= 0; k--) {
    int v = order[k];
    int l = (int)(ch[v - m] & 0xFFFFu), r = (int)(ch[v - m] >> 16);
    const uint64_t* x = l < m ? &I.leaf[(size_t)l * nw] : lab + (size_t)(l - m) * nw;
    const uint64_t* y = r < m ? &I.leaf[(size_t)r * nw] : lab + (size_t)(r - m) * nw;
    uint64_t* z = lab + (size_t)(v - m) * nw;
    for (int w = 0; w < nw; w++) z[w] = x[w] | y[w];
    for (int q : closes[v - m]) z[q >> 6] &= ~(1ull << (q & 63));
  }
  return true;
}

// (cost, size) words of every internal node, on the network sliced by S
void fill_cz(const Inst& I, const uint32_t* ch, const uint64_t* lab, const uint64_t* S, uint32_t* cz) {
  const int m = I.m, nw = I.nw;
  for (int i = 0; i < m - 1; i++) {
    int l = (int)(ch[i] & 0xFFFFu), r = (int)(ch[i] >> 16);
    const uint64_t* x = l < m ? &I.leaf[(size_t)l * nw] : lab + (size_t)(l - m) * nw;
    const uint64_t* y = r < m ? &I.leaf[(size_t)r * nw] : lab + (size_t)(r - m) * nw;
    const uint64_t* z = lab + (size_t)i * nw;
    int Z = 0, K = 0;
    for (int w = 0; w < nw; w++) {
      uint64_t nm = ~S[w], zz = z[w] & nm;
      Z += popc(zz);
      K += popc(x[w] & y[w] & nm & ~zz);
    }
    cz[i] = ((uint32_t)(Z + K) << 16) | (uint32_t)Z;
  }
}

// chunk summaries of n label sets of nw words (bit c: words 2c, 2c+1 not both zero)
void fill_sums(const uint64_t* lab, int n, int nw, uint64_t* out) {
  for (int i = 0; i < n; i++) {
    uint64_t s = 0;
    for (int c = 0; c < nw / 2; c++)
      if (lab[(size_t)i * nw + 2 * c] | lab[(size_t)i * nw + 2 * c + 1]) s |= 1ull << c;
    out[i] = s;
  }
}

// ------------------------------------------------------------------------------------------------
// Host double-precision energies, cost models and the slicer repair (csrc/treesa_gpu.cu:1174-1274)
// ------------------------------------------------------------------------------------------------
struct Models {
  float lpeak, lbw, llaunch;
  int m0, n0, k0;
  float l3launch, lperm2, lcc_bit, lcc_cell, ltc_bit, ltc_pad, ltc_out, lsmall_cell;
  int small_rank;
};
Models make_models(const double* gm_in, const double* hm_in) {  // Runner ctor, :1461-1475
  static const double gm_def[6] = {11.9e15, 1.6e13, 6, 6, 8, 4e-6};
  static const double hm_def[9] = {4e-6, 1.23e13, 5.44e-14, 7.68e-15, 6.37e-14, 2.02e-16, 1.77e-13, 14, 1e-12};
  const double* gm = gm_in ? gm_in : gm_def;
  const double* hm = hm_in ? hm_in : hm_def;
  Models M;
  M.lpeak = (float)log2(gm[0]);
  M.lbw = (float)log2(gm[1]);
  M.m0 = (int)gm[2];
  M.n0 = (int)gm[3];
  M.k0 = (int)gm[4];
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
double gpu_time_d(int B, int M_, int N, int K, const Models& M) {
  double ops = exp2((double)(1 + B + std::max(M_, M.m0) + std::max(N, M.n0) + std::max(K, M.k0)));
  double bits = exp2((double)(B + M_ + K)) + exp2((double)(B + N + K)) + exp2((double)(B + M_ + N));
  return std::max(ops / exp2((double)M.lpeak), bits / exp2((double)M.lbw)) + exp2((double)M.llaunch);
}
double h100_time_d(int B, int M_, int N, int K, const Models& M) {
  auto e = [](float l) { return exp2((double)l); };
  if (B + M_ + N <= M.small_rank) return e(M.lsmall_cell) * exp2((double)(B + M_ + N + K));
  double a = exp2((double)(B + M_ + K)), b = exp2((double)(B + N + K)), c = exp2((double)(B + M_ + N));
  double moved = a + b + c;
  double perm = e(M.lperm2) * (a + b);
  double best = e(M.lcc_bit) * moved + e(M.lcc_cell) * exp2((double)(B + M_ + N + K));
  if (K >= 7 && std::max(M_, N) >= 5) {
    double tc = e(M.ltc_bit) * moved +
                e(M.ltc_pad) * exp2((double)(B + std::max(M_, 6) + std::max(N, 6) + std::max(K, 8))) +
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
  const int nw = I.nw, m = I.m;
  HostE E;
  std::vector<uint64_t> nm(nw, ~0ull);
  if (S)
    for (int w = 0; w < nw; w++) {
      nm[w] = ~S[w];
      E.ns += popc(S[w]);
    }
  for (int i = 0; i < m; i++) {
    int z = 0;
    for (int w = 0; w < nw; w++) z += popc(I.leaf[(size_t)i * nw + w] & nm[w]);
    E.sc = std::max(E.sc, z);
  }
  double mx = -1e300;
  std::vector<double> tcs;
  tcs.reserve(m - 1);
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

// Julia TreeSASlicer rule as a final repair (:1248-1274): while sc > sc_target, slice the label that
// occurs most often among the largest masked tensors (ties: lowest label id).
int greedy_repair(const Inst& I, const uint64_t* lab, uint64_t* S, double sc_target) {
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
        for (int w = 0; w < nw; w++) {
          uint64_t x = a[w] & ~S[w];
          while (x) {
            int b = __builtin_ctzll(x);
            x &= x - 1;
            freq[w * 64 + b]++;
          }
        }
      }
    int best = (int)(std::max_element(freq.begin(), freq.end()) - freq.begin());
    S[best >> 6] |= 1ull << (best & 63);
    added++;
  }
}

float lse_entry(int d) { return (float)log2(1.0 + exp2(-(double)d)); }  // :2075

}  // namespace

// ==================================================================================================
// Session
// ==================================================================================================
struct tsa_session {
  Inst I;
  Layout L{};
  tsa::LaunchPlan plan{};
  // options (owned copies)
  std::vector<float> betas;
  int niters = 0, nchains = 0, scheme = 0, order = 0, eval_every = 1, slicing = 0, slice_moves = 0;
  int par_band = 0, par_follow = 0;  // par-order variants (--par-band, --par-follow)
  // energy of every level (stage 2 appends its levels: --stage2-betas/-niters/-mode, :1758-1764)
  std::vector<int> lmode, lniters;
  int mode0 = 0;     // energy of the first level
  int cur_mode = 0;  // energy of the current level (score() depends on it)
  int slice_every = 1, max_slices = 0, select_sc = 0, verbose = 0, device = 0, rank = 0, world = 1, exp_device = 0;
  double timeout_s = 0;  // > 0: wall-clock limit of a run's level loop (single-GPU runs)
  long long wait_cycles = 1ll << 31;  // limit of the kernels' bounded waits
  int debug_arm_only = 0;             // tests: warp kernels arm the staging barrier without a copy
  double sc_target = 20, sc_weight = 1, trunc_frac = 0.25;
  uint64_t seed = 1;
  uint32_t key0 = 0, key1 = 0;
  Models models{};
  std::vector<uint64_t> S0;
  int chain0 = 0, nglobal = 0;
  // device
  cudaStream_t st = nullptr;
  bool own_stream = false;
  uint8_t *d_rec = nullptr, *d_rec2 = nullptr, *d_init = nullptr;
  uint64_t* d_leaf = nullptr;
  uint64_t* d_leaf_sum = nullptr;
  float *d_lse = nullptr, *d_lc = nullptr;
  int *d_sc = nullptr, *d_ns = nullptr, *d_anc = nullptr, *d_err = nullptr;
  uint8_t* d_best = nullptr;  // level-by-level runs: the owner's device copy of the best record
  unsigned long long* d_stats = nullptr;
  uint32_t* d_scratch = nullptr;  // [nchains][nint] slice-move cost scratch (plan gmeta 2 only)
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEvent_t evk[4] = {nullptr, nullptr, nullptr, nullptr};  // kernel start/end, two level parities
  // level-by-level runs: end of the energy gather, start and end of the population step
  cudaEvent_t evx[3] = {nullptr, nullptr, nullptr};
  double gather_ms = 0, resample_ms = 0;
  double host_s = 0, fetch_s = 0;  // host selection work; best-record fetches (copy or NCCL broadcast)
  uint64_t comm_sent0 = 0, comm_recv0 = 0;  // the communicator's record byte counts when the run began
  cudaEvent_t eve[2] = {nullptr, nullptr};                    // energies of a level on the host
  cudaStream_t cst = nullptr;                                 // energy gathers and best-record copies
  cudaEvent_t evdone[2] = {nullptr, nullptr};                 // a level's kernel has finished (on st)
  cudaEvent_t evfree[2] = {nullptr, nullptr};                 // cst is done with a level's buffers
  float* h_lc = nullptr;                                      // pinned [2][nglobal]
  int *h_sc = nullptr, *h_ns = nullptr;
  uint8_t* h_best = nullptr;                                  // pinned best record
  uint8_t* d_cur = nullptr;                                   // buffer holding the current population
  tsa::Comm* comm = nullptr;
  float h_lse[64];
  double t_init = 0;
  // run state
  bool ran = false;
  double best_score = INFINITY, kernel_ms = 0, t_anneal = 0;
  int best_chain = -1, best_level = -1, nresample = 0;
  uint32_t sweep_ctr = 0;
  std::vector<uint8_t> best;  // record of the best chain (host)
  std::vector<double> trace;
  std::vector<float> lc;
  std::vector<int> sc, ns;
  uint64_t stats[12] = {0};
  uint64_t launches = 0;
  uint64_t h2d = 0, d2h = 0;  // bytes copied between host and device by this session

  ~tsa_session() {
    if (device >= 0) cudaSetDevice(device);
    if (st) cudaStreamSynchronize(st);  // nothing in flight touches the blocks handed back to the cache
    if (cst) cudaStreamSynchronize(cst);
    for (void* p : {(void*)d_rec, (void*)d_rec2, (void*)d_init, (void*)d_leaf, (void*)d_leaf_sum, (void*)d_lse,
                    (void*)d_scratch, (void*)d_lc, (void*)d_sc, (void*)d_ns, (void*)d_anc, (void*)d_err,
                    (void*)d_stats, (void*)h_lc, (void*)h_sc, (void*)h_ns, (void*)h_best, (void*)d_best})
      pool_free(p);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    for (auto& e : evk)
      if (e) cudaEventDestroy(e);
    for (auto& e : evx)
      if (e) cudaEventDestroy(e);
    for (auto& e : eve)
      if (e) cudaEventDestroy(e);
    for (auto& e : evdone)
      if (e) cudaEventDestroy(e);
    for (auto& e : evfree)
      if (e) cudaEventDestroy(e);
    if (cst) cudaStreamDestroy(cst);
    if (own_stream && st) cudaStreamDestroy(st);
    delete comm;
  }

  double score(float l, int s, int n) const {  // :1737-1747
    if (slicing) return (double)n + (double)l + 1000.0 * std::max(0.0, (double)s - sc_target);
    if (select_sc) return 4096.0 * std::max(0.0, (double)s - sc_target) + (double)l;
    if (cur_mode != 0) return energyE(l, s, n);  // the model modes: the log-domain energy
    double tc = (double)l;
    if ((double)s <= sc_target || sc_weight <= 0) return tc;
    double pen = log2(sc_weight) + (double)s + log2(1.0 - exp2(sc_target - (double)s));
    double mx = std::max(tc, pen), mn = std::min(tc, pen);
    return mx + log2(1.0 + exp2(mn - mx));
  }
  double energyE(float l, int s, int n) const {  // :1750-1753
    return (double)n + (double)l + sc_weight * std::max(0.0, (double)s - sc_target);
  }
};

namespace {

int init_device_state(tsa_session* s, const tsa_options* O, char* err, size_t errlen) {
  CKR(cudaSetDevice(s->device));
  if (O->stream) {
    s->st = (cudaStream_t)O->stream;
  } else {
    CKR(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    s->own_stream = true;
  }
  bool model = false;
  for (int md : s->lmode) model = model || md != TSA_MODE_TC;
  if (tsa::plan_sweeps(s->L, s->nchains, s->device, O->kernel_hint, s->order, s->slice_moves, s->par_band, s->par_follow,
                       model ? 1 : 0, &s->plan) !=
      cudaSuccess) {
    set_err(err, errlen, "no sweep kernel for this layout (%d internal nodes, %d label words)", s->L.nint, s->L.nw);
    return TSA_ERR_UNSUPPORTED;
  }
  if (s->plan.gmeta == 2 && (s->slice_moves > 0 || model || s->par_band > 0))
    // per chain: 2 words a node (slice-move costs and model-mode costs, or the band depths)
    CKR(pool_alloc(0, &s->d_scratch, (size_t)s->nchains * 2 * s->L.nint * sizeof(uint32_t)));
  const size_t recb = (size_t)s->L.rec_bytes * s->nchains;
  CKR(pool_alloc(0, &s->d_rec, recb));
  CKR(pool_alloc(0, &s->d_init, recb));
  CKR(pool_alloc(0, &s->d_rec2, recb));
  CKR(pool_alloc(0, &s->d_leaf, s->I.leaf.size() * 8));
  CKR(pool_alloc(0, &s->d_lse, 64 * sizeof(float)));
  CKR(pool_alloc(0, &s->d_lc, 2 * s->nchains * sizeof(float)));
  CKR(pool_alloc(0, &s->d_sc, 2 * s->nchains * sizeof(int)));
  CKR(pool_alloc(0, &s->d_ns, 2 * s->nchains * sizeof(int)));
  CKR(pool_alloc(1, &s->h_lc, 2 * (size_t)s->nglobal * sizeof(float)));
  CKR(pool_alloc(1, &s->h_sc, 2 * (size_t)s->nglobal * sizeof(int)));
  CKR(pool_alloc(1, &s->h_ns, 2 * (size_t)s->nglobal * sizeof(int)));
  CKR(pool_alloc(1, &s->h_best, s->L.rec_bytes));
  CKR(pool_alloc(0, &s->d_best, s->L.rec_bytes));
  for (auto& e : s->evk) CKR(cudaEventCreate(&e));
  for (auto& e : s->evx) CKR(cudaEventCreate(&e));
  for (auto& e : s->eve) CKR(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : s->evdone) CKR(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : s->evfree) CKR(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CKR(cudaStreamCreateWithFlags(&s->cst, cudaStreamNonBlocking));
  CKR(pool_alloc(0, &s->d_anc, s->nchains * sizeof(int)));
  CKR(pool_alloc(0, &s->d_err, sizeof(int)));
  CKR(pool_alloc(0, &s->d_stats, 10 * sizeof(unsigned long long)));
  CKR(cudaEventCreate(&s->ev0));
  CKR(cudaEventCreate(&s->ev1));
  CKR(cudaMemcpyAsync(s->d_leaf, s->I.leaf.data(), s->I.leaf.size() * 8, cudaMemcpyHostToDevice, s->st));
  {
    std::vector<uint64_t> ls(s->I.m, 0);
    if (s->L.sums) fill_sums(s->I.leaf.data(), s->I.m, s->L.nw, ls.data());
    CKR(pool_alloc(0, &s->d_leaf_sum, ls.size() * 8));
    CKR(cudaMemcpy(s->d_leaf_sum, ls.data(), ls.size() * 8, cudaMemcpyHostToDevice));
    s->h2d += ls.size() * 8;
  }
  s->h2d += s->I.leaf.size() * 8 + 64 * sizeof(float) + 64 * sizeof(double);
  for (int d = 0; d < 64; d++) s->h_lse[d] = lse_entry(d);
  CKR(tsa::upload_lse_table(s->h_lse, s->d_lse, s->st));
  return TSA_OK;
}

// Build the initial chain records on the host (init_chains, csrc/treesa_gpu.cu:1585-1630) and upload.
int init_chains(tsa_session* s, const tsa_options* O, char* err, size_t errlen) {
  const Inst& I = s->I;
  const Layout& L = s->L;
  const int nint = L.nint, nw = L.nw, K = O->init_trees ? O->ntrees : 0;
  // distinct start trees: K given trees (chain c from tree c % K), else one random tree per chain
  const int ndist = K > 0 ? std::min(K, s->nglobal) : s->nchains;
  std::vector<uint8_t> host((size_t)L.rec_bytes * (K > 0 ? ndist : s->nchains), 0);
  int bad = 0;
  auto build = [&](const uint32_t* tree, uint8_t* rec) -> bool {
    uint64_t* lab = reinterpret_cast<uint64_t*>(rec);
    uint32_t* ch = reinterpret_cast<uint32_t*>(rec + L.off_ch);
    uint32_t* cz = reinterpret_cast<uint32_t*>(rec + L.off_cz);
    uint64_t* S = reinterpret_cast<uint64_t*>(rec + L.off_S);
    memcpy(ch, tree, (size_t)nint * 4);
    memcpy(S, s->S0.data(), (size_t)nw * 8);
    if (!topo_labels(I, ch, lab)) return false;
    fill_cz(I, ch, lab, S, cz);
    if (L.sums) fill_sums(lab, nint, nw, reinterpret_cast<uint64_t*>(rec + L.off_sum));
    return true;
  };
  if (K > 0) {
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : bad)
    for (int k = 0; k < ndist; k++)
      if (!build(O->init_trees + (size_t)k * nint, &host[(size_t)k * L.rec_bytes])) bad++;
  } else {
#pragma omp parallel for schedule(dynamic, 4) reduction(+ : bad)
    for (int c = 0; c < s->nchains; c++) {
      uint64_t gc = (uint64_t)(s->chain0 + c);
      std::vector<uint32_t> t = random_tree(I.m, splitmix64(s->seed * 1000003ULL + gc));
      if (!build(t.data(), &host[(size_t)c * L.rec_bytes])) bad++;
    }
  }
  if (bad) {
    set_err(err, errlen, "invalid initial tree");
    return TSA_ERR_ARG;
  }
  const size_t bytes = (size_t)L.rec_bytes * s->nchains;
  if (K > 0) {
    // the ndist distinct records go up once and are replicated on the device: chain c <- record
    // (chain0 + c) % K (staged in d_rec2, which the run overwrites before reading)
    std::vector<int> src(s->nchains);
    for (int c = 0; c < s->nchains; c++) src[c] = (s->chain0 + c) % K;
    CKR(cudaMemcpyAsync(s->d_rec2, host.data(), host.size(), cudaMemcpyHostToDevice, s->st));
    CKR(cudaMemcpyAsync(s->d_anc, src.data(), sizeof(int) * s->nchains, cudaMemcpyHostToDevice, s->st));
    s->h2d += host.size() + sizeof(int) * s->nchains;
    CKR(tsa::launch_copy_chains(s->d_rec2, s->d_init, s->d_anc, s->nchains, L.rec_bytes, s->st));
  } else {
    CKR(cudaMemcpyAsync(s->d_init, host.data(), bytes, cudaMemcpyHostToDevice, s->st));
    s->h2d += bytes;
  }
  CKR(cudaMemcpyAsync(s->d_rec, s->d_init, bytes, cudaMemcpyDeviceToDevice, s->st));
  CKR(cudaStreamSynchronize(s->st));
  return TSA_OK;
}

int reset_run_state(tsa_session* s, char* err, size_t errlen) {
  s->ran = false;
  s->cur_mode = s->mode0;
  s->best_score = INFINITY;
  s->best_chain = s->best_level = -1;
  s->nresample = 0;
  s->kernel_ms = 0;
  s->gather_ms = s->resample_ms = 0;
  s->host_s = s->fetch_s = 0;
  if (s->comm) {
    s->comm_sent0 = s->comm->sent_bytes;
    s->comm_recv0 = s->comm->recv_bytes;
  }
  s->t_anneal = 0;
  s->sweep_ctr = 0;
  s->best.clear();
  s->trace.clear();
  s->launches = 0;
  memset(s->stats, 0, sizeof s->stats);
  CKR(cudaMemsetAsync(s->d_stats, 0, 10 * sizeof(unsigned long long), s->st));
  CKR(cudaMemsetAsync(s->d_err, 0, sizeof(int), s->st));
  return TSA_OK;
}

}  // namespace

extern "C" {

int tsa_abi_version(void) { return TSA_ABI_VERSION; }

int tsa_abi_sizes(int32_t* sizes) {
  if (!sizes) return TSA_ERR_ARG;
  sizes[0] = (int32_t)sizeof(tsa_instance);
  sizes[1] = (int32_t)sizeof(tsa_options);
  sizes[2] = (int32_t)sizeof(tsa_result);
  return TSA_OK;
}

int tsa_session_create(const tsa_instance* inst, const tsa_options* O, tsa_session** out, char* err, size_t errlen) {
  if (!out || !O) {
    set_err(err, errlen, "null argument");
    return TSA_ERR_ARG;
  }
  *out = nullptr;
  double t0 = now_s();
  tsa_session* s = new (std::nothrow) tsa_session();
  if (!s) return TSA_ERR_NOMEM;
  s->device = -1;
  int rc = load_inst(inst, s->I, err, errlen);
  if (rc) {
    delete s;
    return rc;
  }
  if (O->mode < TSA_MODE_TC || O->mode > TSA_MODE_H100 ||
      (O->betas2 && O->nbetas2 > 0 && O->mode2 != TSA_MODE_GPU && O->mode2 != TSA_MODE_H100)) {
    set_err(err, errlen, "mode must be tc, gpu or h100, and the stage-2 mode gpu or h100");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->nchains < 1 || O->niters < 0 || O->nbetas < 1 || !O->betas) {
    set_err(err, errlen, "need nchains >= 1, niters >= 0 and at least one beta");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->scheme < 0 || O->scheme > 2 || O->order < 0 || O->order > 1) {
    set_err(err, errlen, "bad scheme or order");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->world_size < 1 || O->rank < 0 || O->rank >= O->world_size) {
    set_err(err, errlen, "bad rank / world_size");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->init_trees && O->ntrees < 1) {
    set_err(err, errlen, "init_trees given with ntrees < 1");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->kernel_hint == 2 && s->I.nw == 1) {  // the CTA-per-chain kernel streams 16-byte chunks
    Inst& J = s->I;
    J.nw = 2;
    J.leaf.assign((size_t)J.m * 2, 0);
    for (int i = 0; i < J.m; i++)
      for (int l : J.ixs[i]) J.leaf[(size_t)i * 2 + (l >> 6)] |= 1ull << (l & 63);
  }
  const Inst& I = s->I;
  s->betas.assign(O->betas, O->betas + O->nbetas);
  if (O->max_levels > 0 && (int)s->betas.size() > O->max_levels) s->betas.resize(O->max_levels);
  s->niters = O->niters;
  s->lmode.assign(s->betas.size(), O->mode);
  s->lniters.assign(s->betas.size(), O->niters);
  if (O->betas2 && O->nbetas2 > 0)
    for (int k = 0; k < O->nbetas2; k++) {
      s->betas.push_back(O->betas2[k]);
      s->lmode.push_back(O->mode2);
      s->lniters.push_back(O->niters2 > 0 ? O->niters2 : O->niters);
    }
  s->mode0 = s->cur_mode = O->mode;
  s->nchains = O->nchains;
  s->scheme = O->scheme;
  s->order = O->order;
  s->eval_every = std::max(1, O->eval_every);
  s->slicing = O->slicing ? 1 : 0;
  s->slice_moves = O->slicing ? std::max(0, O->slice_moves) : 0;
  s->slice_every = std::max(1, O->slice_every);
  s->max_slices = O->max_slices > 0 ? O->max_slices : I.nlab;
  s->select_sc = O->select_sc ? 1 : 0;
  s->verbose = O->verbose;
  if (O->par_band < 0 || O->par_band == 1 || O->par_band > 16) {
    set_err(err, errlen, "--par-band L: 0 (off) or 2..16");
    delete s;
    return TSA_ERR_ARG;
  }
  s->par_band = O->order == TSA_ORDER_PAR ? O->par_band : 0;
  s->par_follow = O->order == TSA_ORDER_PAR && O->par_follow ? 1 : 0;
  if (!(O->timeout_s >= 0.0f) || std::isinf(O->timeout_s)) {
    set_err(err, errlen, "timeout_s must be a finite number >= 0");
    delete s;
    return TSA_ERR_ARG;
  }
  s->timeout_s = O->timeout_s;
  if (O->wait_log2 != 0 && (O->wait_log2 < 10 || O->wait_log2 > 31)) {
    set_err(err, errlen, "wait_log2 must be 0 (default, 2^31 cycles) or 10..31");
    delete s;
    return TSA_ERR_ARG;
  }
  s->wait_cycles = 1ll << (O->wait_log2 ? O->wait_log2 : 31);
  if (O->debug_flags & ~TSA_DEBUG_ARM_ONLY) {
    set_err(err, errlen, "unknown debug_flags bits 0x%x", (unsigned)(O->debug_flags & ~TSA_DEBUG_ARM_ONLY));
    delete s;
    return TSA_ERR_ARG;
  }
  s->debug_arm_only = (O->debug_flags & TSA_DEBUG_ARM_ONLY) ? 1 : 0;
  bool model = false;
  for (int md : s->lmode) model = model || md != TSA_MODE_TC;
  if (O->kernel_hint == 3 && (s->par_band || s->par_follow || model)) {
    set_err(err, errlen, "kernel_hint 3 (two warps per chain) runs plain par order in mode tc");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->kernel_hint < 0 || O->kernel_hint > 4) {
    set_err(err, errlen, "kernel_hint must be 0 (auto), 1 (warp), 2 (block), 3 (pair of warps) or 4 (pair of CTAs)");
    delete s;
    return TSA_ERR_ARG;
  }
  if (O->exp_mode < 0 || O->exp_mode > 1) {
    set_err(err, errlen, "exp_mode must be 0 (host libm) or 1 (device expf)");
    delete s;
    return TSA_ERR_ARG;
  }
  s->exp_device = O->exp_mode;
  s->sc_target = O->sc_target;
  s->sc_weight = O->sc_weight;
  s->trunc_frac = O->trunc_frac;
  s->seed = O->seed;
  uint64_t k = splitmix64(O->seed);
  s->key0 = (uint32_t)k;
  s->key1 = (uint32_t)(k >> 32);
  s->models = make_models(O->gpu_model, O->h100_model);
  s->rank = O->rank;
  s->world = O->world_size;
  s->chain0 = O->rank * O->nchains;
  s->nglobal = O->nchains * O->world_size;
  s->device = O->device;
  // layout
  Layout& L = s->L;
  L.m = I.m;
  L.nint = I.m - 1;
  L.nw = I.nw;
  uint32_t lab_bytes = (uint32_t)L.nint * (uint32_t)L.nw * 8u;
  L.off_ch = rup(lab_bytes, 16);
  L.off_cz = L.off_ch + rup((uint32_t)L.nint * 4u, 16);
  L.off_S = L.off_cz + rup((uint32_t)L.nint * 4u, 16);
  // chunk summaries (one u64 per node: 16-byte chunk c nonzero) for wide sets of 32..128 words
  L.sums = (L.nw >= 32 && L.nw <= 128) ? 1 : 0;
  L.off_sum = rup(L.off_S + (uint32_t)L.nw * 8u, 16);
  L.rec_bytes = rup(L.off_sum + (L.sums ? (uint32_t)L.nint * 8u : 0u), 128);
  s->S0.assign(L.nw, 0);
  for (int j = 0; j < O->ninit_slices; j++) {
    int l = O->init_slices[j];
    if (l < 0 || l >= I.nlab) {
      set_err(err, errlen, "bad init_slices label");
      delete s;
      return TSA_ERR_ARG;
    }
    s->S0[l >> 6] |= 1ull << (l & 63);
    s->slicing = 1;
  }
  if (O->world_size > 1) {
    rc = tsa::comm_create(O->nccl_id, O->rank, O->world_size, O->device, &s->comm, err, errlen);
    if (rc) {
      delete s;
      return rc;
    }
  }
  rc = init_device_state(s, O, err, errlen);
  if (rc == TSA_OK) rc = init_chains(s, O, err, errlen);
  if (rc == TSA_OK) rc = reset_run_state(s, err, errlen);
  if (rc) {
    delete s;
    return rc;
  }
  s->t_init = now_s() - t0;
  *out = s;
  return TSA_OK;
}

void tsa_session_destroy(tsa_session* s) { delete s; }

int tsa_session_reset(tsa_session* s, char* err, size_t errlen) {
  if (!s) return TSA_ERR_ARG;
  CKR(cudaSetDevice(s->device));
  CKR(cudaMemcpyAsync(s->d_rec, s->d_init, (size_t)s->L.rec_bytes * s->nchains, cudaMemcpyDeviceToDevice, s->st));
  s->d_cur = s->d_rec;
  int rc = reset_run_state(s, err, errlen);
  if (rc) return rc;
  CKR(cudaStreamSynchronize(s->st));
  return TSA_OK;
}

// The beta-level loop (run_anneal, csrc/treesa_gpu.cu:1789-1877).  Best-of-N runs of the warp kernel are
// pipelined: level l reads one record buffer and writes the other, its energies go to pinned host memory,
// and the host scores level l (and, when the best improves, copies the best record out of level l's
// output buffer) while level l+1 runs; level l+2, which overwrites that buffer, is enqueued after the
// copy.  Population schemes need level l's energies before level l+1 and run level by level.
int tsa_session_run(tsa_session* s, char* err, size_t errlen) {
  if (!s) return TSA_ERR_ARG;
  if (s->ran) {
    set_err(err, errlen, "session already ran: call tsa_session_reset first");
    return TSA_ERR_ARG;
  }
  CKR(cudaSetDevice(s->device));
  const int nch = s->nchains, ng = s->nglobal;
  const size_t nlev = s->betas.size();
  const uint32_t rb = s->L.rec_bytes;
  double t0 = now_s();
  s->lc.assign(nch, 0.f);
  s->sc.assign(nch, 0);
  s->ns.assign(nch, 0);
  std::vector<int> family(ng), nfam(ng);
  std::iota(family.begin(), family.end(), 0);
  std::mt19937_64 hrng(splitmix64(s->seed + 777));
  float beta_last = s->betas[0];
  bool staged = false;
  for (int md : s->lmode) staged = staged || md != s->lmode[0];
  const bool pipelined = s->scheme == TSA_SCHEME_INDEP && s->plan.kind != tsa::K_BLOCK && !staged;
  tsa::SweepArgs a{};
  a.L = s->L;
  a.leaf = s->d_leaf;
  a.nchains = nch;
  a.chain0 = s->chain0;
  a.order = s->order;
  a.nsweeps = s->niters;
  a.sc_target = (float)s->sc_target;
  a.sc_weight = (float)s->sc_weight;
  a.key0 = s->key0;
  a.key1 = s->key1;
  a.slicing = s->slicing;
  a.exp_device = s->exp_device;
  a.leaf_sc = s->I.leaf_sc;
  a.slice_moves = s->slice_moves;
  a.par_band = s->par_band;
  a.par_follow = s->par_follow;
  a.mode = s->cur_mode;
  {
    const Models& M = s->models;
    a.mp = tsa::ModelParams{M.lpeak,    M.lbw,    M.llaunch, M.m0,      M.n0,      M.k0,     M.l3launch, M.lperm2,
                            M.lcc_bit,  M.lcc_cell, M.ltc_bit, M.ltc_pad, M.ltc_out, M.lsmall_cell, M.small_rank};
  }
  a.slice_every = s->slice_every;
  a.max_slices = s->max_slices;
  a.stats = s->d_stats;
  a.err = s->d_err;
  a.wait_cycles = s->wait_cycles;
  a.debug_arm_only = s->debug_arm_only;
  a.lse_tab = s->d_lse;
  a.leaf_sum = s->d_leaf_sum;
  a.scratch = s->d_scratch;
  s->best.resize(rb);
  // every chain's score and energy of the evaluated level (the selection step reuses the energies),
  // computed by a few host threads for large populations, then reduced in chain order
  std::vector<double> SV(ng), EV(ng);
  const int hthreads = ng >= 2048 ? std::min(4, std::max(1, omp_get_num_procs())) : 1;
  // host side of one evaluated level: best tracking and trace
  auto process = [&](size_t lev, const float* glc, const int* gsc, const int* gns, int* improved) {
#pragma omp parallel for num_threads(hthreads) schedule(static)
    for (int c = 0; c < ng; c++) {
      SV[c] = s->score(glc[c], gsc[c], gns[c]);
      EV[c] = s->energyE(glc[c], gsc[c], gns[c]);
    }
    int bi = 0;
    double bs = INFINITY, meanE = 0, meanNs = 0;
    for (int c = 0; c < ng; c++) {
      if (SV[c] < bs) {
        bs = SV[c];
        bi = c;
      }
      meanE += EV[c];
      meanNs += gns[c];
    }
    meanE /= ng;
    meanNs /= ng;
    *improved = -1;
    if (bs < s->best_score) {
      s->best_score = bs;
      s->best_chain = bi;
      s->best_level = (int)lev;
      *improved = bi;
    }
    std::fill(nfam.begin(), nfam.end(), 0);
    int nf = 0;
    for (int c = 0; c < ng; c++)
      if (nfam[family[c]]++ == 0) nf++;
    double row[10] = {now_s() - t0, (double)lev, (double)s->betas[lev], (double)glc[bi], (double)gsc[bi], meanE,
                      (double)nf, (double)s->cur_mode, (double)gns[bi], meanNs};
    s->trace.insert(s->trace.end(), row, row + 10);
    if (s->verbose && (lev % 25 == 0 || lev + 1 == nlev))
      fprintf(stderr, "lev %4zu beta %7.3f  best(l2cost/slice %.3f sc %d |S| %d)  meanE %.3f  families %d  t=%.2fs\n",
              lev, s->betas[lev], (double)glc[bi], gsc[bi], gns[bi], meanE, nf, now_s() - t0);
  };
  // Best-of-N over several ranks needs no exchange per level: every rank scores its own chains and keeps
  // its own best record (process_local), and one exchange after the last level (reduce_local) picks the
  // global best and rebuilds the trace.  The first strict improvement in (level, chain) order is the
  // smallest (score, level, chain), so the winner is the chain a single-rank run of the whole population
  // picks.  Population schemes and staged runs (whose incumbent is rescored at the stage switch) gather
  // every chain's energies after each evaluated level.
  const bool local = s->world > 1 && s->scheme == TSA_SCHEME_INDEP && !staged;
  constexpr int kLS = 9;     // per evaluated level: t, level, best score, its global chain, lc, sc, |S|, sum E, sum |S|
  std::vector<double> lsum;  // this rank's summaries of the evaluated levels
  auto process_local = [&](size_t lev, int q, int* improved) {
    const size_t off = (size_t)q * ng + (size_t)s->rank * nch;
    const float* lc = s->h_lc + off;
    const int *sc = s->h_sc + off, *ns = s->h_ns + off;
    int bi = 0;
    double bs = INFINITY, sumE = 0, sumNs = 0;
    for (int c = 0; c < nch; c++) {
      double sv = s->score(lc[c], sc[c], ns[c]);
      if (sv < bs) {
        bs = sv;
        bi = c;
      }
      sumE += s->energyE(lc[c], sc[c], ns[c]);
      sumNs += ns[c];
    }
    const int g = s->rank * nch + bi;
    *improved = -1;
    if (bs < s->best_score) {
      s->best_score = bs;
      s->best_chain = g;
      s->best_level = (int)lev;
      *improved = g;
    }
    const double row[kLS] = {now_s() - t0, (double)lev, bs, (double)g, (double)lc[bi], (double)sc[bi],
                             (double)ns[bi], sumE, sumNs};
    lsum.insert(lsum.end(), row, row + kLS);
  };
  auto reduce_local = [&]() -> int {
    const int n = 3 + (int)lsum.size();
    std::vector<double> mine(n), all((size_t)n * s->world);
    mine[0] = s->best_score;
    mine[1] = s->best_level;
    mine[2] = s->best_chain;
    std::copy(lsum.begin(), lsum.end(), mine.begin() + 3);
    int rc2 = s->comm->allgather_host(mine.data(), n, all.data(), s->st, err, errlen);
    if (rc2) return rc2;
    int owner = -1;
    for (int r = 0; r < s->world; r++) {
      const double* m = &all[(size_t)r * n];
      if (m[2] < 0) continue;
      const double* o = owner >= 0 ? &all[(size_t)owner * n] : nullptr;
      if (!o || std::make_tuple(m[0], m[1], m[2]) < std::make_tuple(o[0], o[1], o[2])) owner = r;
    }
    if (owner >= 0) {
      const double* m = &all[(size_t)owner * n];
      s->best_score = m[0];
      s->best_level = (int)m[1];
      s->best_chain = (int)m[2];
      if ((rc2 = s->comm->bcast_host(s->h_best, rb, owner, s->st, err, errlen))) return rc2;
      if (s->rank != owner) s->d2h += rb;
    }
    const int nev = (int)lsum.size() / kLS;
    for (int e = 0; e < nev; e++) {
      auto at = [&](int r) { return &all[(size_t)r * n + 3 + (size_t)e * kLS]; };
      int br = 0;
      double sE = 0, sN = 0;
      for (int r = 0; r < s->world; r++) {
        if (at(r)[2] < at(br)[2]) br = r;
        sE += at(r)[7];
        sN += at(r)[8];
      }
      const double* b = at(br);
      const size_t lev = (size_t)b[1];
      const double row[10] = {at(0)[0], b[1], (double)s->betas[lev], b[4], b[5], sE / ng, (double)ng,
                              (double)s->cur_mode, b[6], sN / ng};
      s->trace.insert(s->trace.end(), row, row + 10);
      if (s->verbose && (lev % 25 == 0 || lev + 1 == nlev))
        fprintf(stderr, "lev %4zu beta %7.3f  best(l2cost/slice %.3f sc %d |S| %d)  meanE %.3f  families %d  t=%.2fs\n",
                lev, s->betas[lev], b[4], (int)b[5], (int)b[6], sE / ng, ng, at(0)[0]);
    }
    return TSA_OK;
  };
  // enqueue on stream cs: energies of this level into pinned host slot q (every rank's with the gather,
  // else this rank's, at its place in the slot)
  auto gather = [&](int q, cudaStream_t cs) -> int {
    if (s->world > 1 && !local)
      return s->comm->allgather_energies(s->d_lc + (size_t)q * nch, s->d_sc + (size_t)q * nch,
                                         s->d_ns + (size_t)q * nch, nch, s->h_lc + (size_t)q * ng,
                                         s->h_sc + (size_t)q * ng, s->h_ns + (size_t)q * ng, cs, err, errlen);
    const size_t off = (size_t)q * ng + (size_t)s->rank * nch;
    CKR(cudaMemcpyAsync(s->h_lc + off, s->d_lc + (size_t)q * nch, nch * sizeof(float), cudaMemcpyDeviceToHost, cs));
    CKR(cudaMemcpyAsync(s->h_sc + off, s->d_sc + (size_t)q * nch, nch * sizeof(int), cudaMemcpyDeviceToHost, cs));
    CKR(cudaMemcpyAsync(s->h_ns + off, s->d_ns + (size_t)q * nch, nch * sizeof(int), cudaMemcpyDeviceToHost, cs));
    return TSA_OK;
  };
  // enqueue on stream cs: copy global chain g's record out of buffer buf into the pinned best record
  // (broadcast from its owner, or, scoring locally, a copy of this rank's own chain)
  auto fetch_best = [&](int g, uint8_t* buf, cudaStream_t cs) -> int {
    s->d2h += rb;
    if (s->world > 1 && !local)
      return s->comm->fetch_record(buf + (size_t)(g % nch) * rb, rb, g / nch, s->h_best, cs, err, errlen);
    CKR(cudaMemcpyAsync(s->h_best, buf + (size_t)(g - s->rank * nch) * rb, rb, cudaMemcpyDeviceToHost, cs));
    return TSA_OK;
  };
  // Level-by-level runs keep an improved best record on its owner's device (a device copy, no wait) and
  // bring it to the host only when the host needs it (a stage switch, the end of the run): one transfer
  // instead of a broadcast and a synchronisation per improvement.  With local scoring every rank keeps
  // its own best and copies it to the host alone (reduce_local then broadcasts the winner's).
  bool best_pending = false;
  int best_owner = 0;
  auto keep_best = [&](int g) -> int {
    best_owner = s->world > 1 && !local ? g / nch : s->rank;
    best_pending = true;
    if (best_owner == s->rank)
      CKR(cudaMemcpyAsync(s->d_best, s->d_cur + (size_t)(g - s->rank * nch) * rb, rb, cudaMemcpyDeviceToDevice,
                          s->st));
    return TSA_OK;
  };
  auto materialize_best = [&]() -> int {
    if (!best_pending) return TSA_OK;
    const double th = now_s();
    s->d2h += rb;
    if (s->world > 1 && !local) {  // a collective: every rank reaches it at the same point of the run
      const int r = s->comm->fetch_record(s->d_best, rb, best_owner, s->h_best, s->st, err, errlen);
      if (r) return r;
    } else {
      CKR(cudaMemcpyAsync(s->h_best, s->d_best, rb, cudaMemcpyDeviceToHost, s->st));
    }
    CKR(cudaStreamSynchronize(s->st));
    best_pending = false;
    s->fetch_s += now_s() - th;
    return TSA_OK;
  };
  auto check_err = [&]() -> int {
    int herr = 0;
    CKR(cudaMemcpy(&herr, s->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
      set_err(err, errlen, "a bounded device wait timed out (code %d)", herr);
      return TSA_ERR_TIMEOUT;
    }
    return TSA_OK;
  };
  // the reference driver's `timeout` (subprocess.run, treesa_gpu/driver.py:305), checked between levels.  A
  // rank of a multi-GPU run never stops alone: its peers would wait for it in their next collective.
  auto past_deadline = [&](size_t lev) -> bool {
    if (s->timeout_s <= 0 || s->world > 1 || now_s() - t0 <= s->timeout_s) return false;
    set_err(err, errlen, "run stopped at its time limit of %g s before level %zu of %zu", s->timeout_s, lev, nlev);
    return true;
  };
  int rc = TSA_OK;
  bool resample_pending = false;  // a population step's events await their elapsed time
  uint8_t* buf[2] = {s->d_rec, s->d_rec2};
  if (pipelined) {
    long pend = -1;  // evaluated level whose energies are in flight
    for (size_t lev = 0; lev <= nlev && rc == TSA_OK; lev++) {
      if (lev < nlev && past_deadline(lev)) {
        rc = TSA_ERR_DEADLINE;
        break;
      }
      if (lev < nlev) {
        const int q = (int)(lev & 1);
        if (lev >= 2) {  // the timing events of level lev-2 are reused now
          CKR(cudaEventSynchronize(s->evk[2 * q + 1]));
          float ms = 0;
          CKR(cudaEventElapsedTime(&ms, s->evk[2 * q], s->evk[2 * q + 1]));
          s->kernel_ms += ms;
        }
        a.recs = buf[q];
        a.recs_out = buf[q ^ 1];
        a.beta = s->betas[lev];
        a.sweep0 = s->sweep_ctr;
        a.out_lc = s->d_lc + (size_t)q * nch;
        a.out_sc = s->d_sc + (size_t)q * nch;
        a.out_ns = s->d_ns + (size_t)q * nch;
        // level lev-2's energies and output records (this level's slot q) must be off the device first
        if (lev >= 2) CKR(cudaStreamWaitEvent(s->st, s->evfree[q], 0));
        CKR(cudaEventRecord(s->evk[2 * q], s->st));
        CKR(tsa::launch_sweeps(a, s->plan, s->st));
        CKR(cudaEventRecord(s->evk[2 * q + 1], s->st));
        CKR(cudaEventRecord(s->evdone[q], s->st));
        s->launches++;
        s->sweep_ctr += (uint32_t)s->niters;
      }
      if (pend >= 0) {
        const int q = (int)(pend & 1);
        CKR(cudaEventSynchronize(s->eve[q]));
        int improved;
        if (local)
          process_local((size_t)pend, q, &improved);
        else
          process((size_t)pend, s->h_lc + (size_t)q * ng, s->h_sc + (size_t)q * ng, s->h_ns + (size_t)q * ng,
                  &improved);
        if (improved >= 0) rc = fetch_best(improved, buf[q ^ 1], s->cst);  // level pend's output buffer
        if (rc == TSA_OK) CKR(cudaEventRecord(s->evfree[q], s->cst));
        pend = -1;
      }
      if (lev < nlev && rc == TSA_OK) {
        const int q = (int)(lev & 1);
        const bool eval = (int)(lev % s->eval_every) == s->eval_every - 1 || lev + 1 == nlev;
        CKR(cudaStreamWaitEvent(s->cst, s->evdone[q], 0));
        if (eval) {
          rc = gather(q, s->cst);
          if (rc == TSA_OK) {
            CKR(cudaEventRecord(s->eve[q], s->cst));
            s->d2h += (size_t)nch * 12;
            pend = (long)lev;
          }
        } else {
          CKR(cudaEventRecord(s->evfree[q], s->cst));
        }
      }
    }
    for (size_t lev = nlev >= 2 ? nlev - 2 : 0; lev < nlev && rc == TSA_OK; lev++) {  // the last two levels
      const int q = (int)(lev & 1);
      CKR(cudaEventSynchronize(s->evk[2 * q + 1]));
      float ms = 0;
      CKR(cudaEventElapsedTime(&ms, s->evk[2 * q], s->evk[2 * q + 1]));
      s->kernel_ms += ms;
    }
    s->d_cur = buf[nlev & 1];
  } else {
    s->d_cur = s->d_rec;
    for (size_t lev = 0; lev < nlev && rc == TSA_OK; lev++) {
      if (past_deadline(lev)) {
        rc = TSA_ERR_DEADLINE;
        break;
      }
      if (s->lmode[lev] != s->cur_mode) {
        // stage switch (:1789-1799): the incumbent, rescored in the new energy, stays the best until beaten
        s->cur_mode = s->lmode[lev];
        if (s->best_chain >= 0) {
          if ((rc = materialize_best())) break;
          const uint8_t* br = s->h_best;
          HostE H1 = host_energy(s->I, s->models, reinterpret_cast<const uint64_t*>(br),
                                 reinterpret_cast<const uint32_t*>(br + s->L.off_ch),
                                 s->slicing ? reinterpret_cast<const uint64_t*>(br + s->L.off_S) : nullptr);
          s->best_score = s->score((float)log2(s->cur_mode == TSA_MODE_GPU ? H1.time : H1.time2), H1.sc, H1.ns);
        }
        beta_last = s->betas[lev];
      }
      a.mode = s->cur_mode;
      a.nsweeps = s->lniters[lev];
      a.recs = s->d_cur;
      a.recs_out = s->d_cur;
      a.beta = s->betas[lev];
      a.sweep0 = s->sweep_ctr;
      a.out_lc = s->d_lc;
      a.out_sc = s->d_sc;
      a.out_ns = s->d_ns;
      CKR(cudaEventRecord(s->evk[0], s->st));
      CKR(tsa::launch_sweeps(a, s->plan, s->st));
      CKR(cudaEventRecord(s->evk[1], s->st));
      s->launches++;
      s->sweep_ctr += (uint32_t)s->lniters[lev];
      const bool last = lev + 1 == nlev;
      const bool switching = !last && s->lmode[lev + 1] != s->cur_mode;  // no population step across it
      const bool eval = (int)(lev % s->eval_every) == s->eval_every - 1 || last || switching;
      if (eval) {
        rc = gather(0, s->st);
        if (rc) break;
        s->d2h += (size_t)nch * 12;
        CKR(cudaEventRecord(s->evx[0], s->st));
      }
      CKR(cudaStreamSynchronize(s->st));
      float ms = 0;
      CKR(cudaEventElapsedTime(&ms, s->evk[0], s->evk[1]));
      s->kernel_ms += ms;
      if (resample_pending) {  // the previous level's population step, complete by now
        CKR(cudaEventElapsedTime(&ms, s->evx[1], s->evx[2]));
        s->resample_ms += ms;
        resample_pending = false;
      }
      if (eval) {
        CKR(cudaEventElapsedTime(&ms, s->evk[1], s->evx[0]));
        s->gather_ms += ms;
      }
      if ((rc = check_err())) break;
      if (!eval) continue;
      const float* glc = s->h_lc;
      const int *gsc = s->h_sc, *gns = s->h_ns;
      int improved;
      double th = now_s();
      if (local)
        process_local(lev, 0, &improved);
      else
        process(lev, glc, gsc, gns, &improved);
      s->host_s += now_s() - th;
      if (improved >= 0 && (rc = keep_best(improved))) break;
      if (last || switching || s->scheme == TSA_SCHEME_INDEP) continue;
      th = now_s();
      std::vector<int> anc(ng);
      const std::vector<double>& E = EV;  // every chain's energy at this level (process)
      if (s->scheme == TSA_SCHEME_PA) {  // :1837-1856
        double db = s->betas[lev + 1] - beta_last;
        beta_last = s->betas[lev + 1];
        std::vector<double> w(ng);
        double Emin = INFINITY;
        for (int c = 0; c < ng; c++) Emin = std::min(Emin, E[c]);
#pragma omp parallel for num_threads(hthreads) schedule(static)
        for (int c = 0; c < ng; c++) w[c] = exp(-db * (E[c] - Emin));
        double wsum = 0;
        for (int c = 0; c < ng; c++) wsum += w[c];
        double u = std::uniform_real_distribution<double>(0, 1)(hrng), acc = 0;
        int j = 0;
        for (int c = 0; c < ng; c++) {
          acc += w[c] / wsum * ng;
          while (j < ng && j + u < acc) anc[j++] = c;
        }
        while (j < ng) anc[j++] = ng - 1;
      } else {  // truncation, :1857-1869
        std::vector<int> idx(ng);
        std::iota(idx.begin(), idx.end(), 0);
        std::sort(idx.begin(), idx.end(), [&](int x, int y) { return E[x] < E[y]; });
        std::iota(anc.begin(), anc.end(), 0);
        int nrep = (int)(s->trunc_frac * ng);
        for (int q = 0; q < nrep; q++) anc[idx[ng - 1 - q]] = idx[q];
      }
      uint8_t* other = s->d_cur == s->d_rec ? s->d_rec2 : s->d_rec;
      s->host_s += now_s() - th;
      CKR(cudaEventRecord(s->evx[1], s->st));
      if (s->world > 1) {
        rc = s->comm->resample(anc.data(), s->d_cur, other, s->d_anc, nch, rb, s->st, err, errlen);
        if (rc) break;
      } else {
        CKR(cudaMemcpyAsync(s->d_anc, anc.data(), nch * sizeof(int), cudaMemcpyHostToDevice, s->st));
        s->h2d += nch * sizeof(int);
        CKR(tsa::launch_copy_chains(s->d_cur, other, s->d_anc, nch, rb, s->st));
      }
      CKR(cudaEventRecord(s->evx[2], s->st));
      resample_pending = true;
      s->d_cur = other;
      std::vector<int> nfm(ng);
      for (int c = 0; c < ng; c++) nfm[c] = family[anc[c]];
      family.swap(nfm);
      s->nresample++;
    }
  }
  if (rc) return rc;
  CKR(cudaStreamSynchronize(s->st));
  CKR(cudaStreamSynchronize(s->cst));
  if (resample_pending) {
    float ms = 0;
    CKR(cudaEventElapsedTime(&ms, s->evx[1], s->evx[2]));
    s->resample_ms += ms;
  }
  if ((rc = check_err())) return rc;
  if ((rc = materialize_best())) return rc;
  if (local && (rc = reduce_local())) return rc;
  memcpy(s->best.data(), s->h_best, rb);
  // the energies of the last level, this rank's chains
  {
    const int q = pipelined ? (int)((nlev - 1) & 1) : 0;
    const size_t off = (size_t)q * ng + (size_t)s->rank * nch;
    memcpy(s->lc.data(), s->h_lc + off, nch * sizeof(float));
    memcpy(s->sc.data(), s->h_sc + off, nch * sizeof(int));
    memcpy(s->ns.data(), s->h_ns + off, nch * sizeof(int));
  }
  unsigned long long st[10];
  CKR(cudaMemcpy(st, s->d_stats, sizeof st, cudaMemcpyDeviceToHost));
  s->d2h += sizeof st;
  for (int q = 0; q < 10; q++) s->stats[q] = st[q];
  s->stats[7] = s->launches;
  if (s->world > 1) {
    rc = s->comm->sum_u64(s->stats, 10, s->st, err, errlen);
    if (rc) return rc;
    s->stats[7] = s->launches;
  }
  s->stats[10] = s->h2d;
  s->stats[11] = s->d2h;
  s->t_anneal = now_s() - t0;
  s->ran = true;
  return TSA_OK;
}

// Finalize (csrc/treesa_gpu.cu:1878-1919): labels check, greedy repair, host energies.
int tsa_session_result(tsa_session* s, tsa_result* res, char* err, size_t errlen) {
  if (!s || !res) return TSA_ERR_ARG;
  memset(res, 0, sizeof *res);
  if (!s->ran || s->best_chain < 0) {
    set_err(err, errlen, "no completed run in this session");
    return TSA_ERR_ARG;
  }
  const Inst& I = s->I;
  const Layout& L = s->L;
  const int nint = L.nint, nw = L.nw;
  const uint64_t* blab = reinterpret_cast<const uint64_t*>(s->best.data());
  const uint32_t* bch = reinterpret_cast<const uint32_t*>(s->best.data() + L.off_ch);
  std::vector<uint64_t> S(reinterpret_cast<const uint64_t*>(s->best.data() + L.off_S),
                          reinterpret_cast<const uint64_t*>(s->best.data() + L.off_S) + nw);
  std::vector<uint64_t> lab2((size_t)nint * nw, 0);
  bool valid = topo_labels(I, bch, lab2.data());
  bool labels_ok = valid && memcmp(lab2.data(), blab, lab2.size() * 8) == 0;
  int n_repair = 0;
  if (s->slicing && valid) n_repair = greedy_repair(I, lab2.data(), S.data(), s->sc_target);
  HostE HE = host_energy(I, s->models, lab2.data(), bch, s->slicing ? S.data() : nullptr);
  res->m = I.m;
  res->tree = (uint32_t*)malloc(sizeof(uint32_t) * std::max(1, nint));
  memcpy(res->tree, bch, (size_t)nint * 4);
  std::vector<int> sl;
  if (s->slicing)
    for (int l = 0; l < I.nlab; l++)
      if (S[l >> 6] >> (l & 63) & 1ull) sl.push_back(l);
  res->nsliced = (int)sl.size();
  res->sliced = (int32_t*)malloc(sizeof(int32_t) * std::max<size_t>(1, sl.size()));
  if (!sl.empty()) memcpy(res->sliced, sl.data(), sl.size() * 4);
  res->tc = HE.tc;
  res->sc = HE.sc;
  res->gpu_time = HE.time;
  res->h100_time = HE.time2;
  res->valid = valid;
  res->labels_ok = labels_ok;
  res->best_chain = s->best_chain;
  res->slicing = s->slicing;
  res->n_repair = n_repair;
  res->tc_total = HE.tc + HE.ns;
  res->gpu_time_total = HE.time * exp2((double)HE.ns);
  res->h100_time_total = HE.time2 * exp2((double)HE.ns);
  res->t_anneal = s->t_anneal;
  res->t_init = s->t_init;
  res->kernel_s = s->kernel_ms / 1e3;
  res->proposals = s->stats[0];
  res->accepts = s->stats[1];
  res->warp_steps = s->stats[2];
  res->node_visits = (uint64_t)s->sweep_ctr * (uint64_t)s->nglobal * (uint64_t)nint;
  res->slice_proposals = s->stats[4];
  res->slice_accepts = s->stats[5];
  res->busy_lanes = s->stats[6];
  res->nchains = s->nglobal;
  res->niters = s->niters;
  res->nlevels = (int)s->betas.size();
  res->total_sweeps = (int)s->sweep_ctr;
  res->W = 0;
  res->nw = nw;
  res->scheme = s->scheme;
  res->mode = s->cur_mode;
  res->nresample = s->nresample;
  res->order = s->order;
  res->ntrace = (int)(s->trace.size() / 10);
  res->trace = (double*)malloc(sizeof(double) * std::max<size_t>(1, s->trace.size()));
  if (!s->trace.empty()) memcpy(res->trace, s->trace.data(), s->trace.size() * 8);
  snprintf(res->kernel, sizeof res->kernel, "%s",
           s->plan.kind == tsa::K_WARP   ? "warp_smem"
           : s->plan.kind == tsa::K_PAIR ? "pair_smem"
           : s->plan.cluster == 2        ? "cta_pair_hbm"
           : s->plan.gmeta == 2          ? "block_hbm_gmeta_scan"
           : s->plan.gmeta               ? "block_hbm_gmeta"
                                         : "block_hbm");
  res->h2d_bytes = s->h2d;
  res->d2h_bytes = s->d2h;
  return valid && labels_ok ? TSA_OK : TSA_ERR_INVALID;
}

void tsa_result_free(tsa_result* r) {
  if (!r) return;
  free(r->tree);
  free(r->sliced);
  free(r->trace);
  r->tree = nullptr;
  r->sliced = nullptr;
  r->trace = nullptr;
}

int tsa_run(const tsa_instance* inst, const tsa_options* opt, tsa_result* res, char* err, size_t errlen) {
  if (res) memset(res, 0, sizeof *res);
  if (err && errlen) err[0] = 0;
  tsa_session* s = nullptr;
  int rc = tsa_session_create(inst, opt, &s, err, errlen);
  if (rc) return rc;
  rc = tsa_session_run(s, err, errlen);
  if (rc == TSA_OK) rc = tsa_session_result(s, res, err, errlen);
  if (rc == TSA_ERR_INVALID) set_err(err, errlen, "final tree invalid or labels mismatch");
  tsa_session_destroy(s);
  return rc;
}

int tsa_session_timing(tsa_session* s, double* t8) {
  if (!s || !t8) return TSA_ERR_ARG;
  double* t6 = t8;
  t8[6] = t8[7] = 0;
  t6[0] = s->kernel_ms / 1e3;
  t6[1] = s->gather_ms / 1e3;
  t6[2] = s->resample_ms / 1e3;
  t6[3] = s->t_anneal;
  t6[4] = s->host_s;
  t6[5] = s->fetch_s;
  if (s->comm) {
    t8[6] = (double)(s->comm->sent_bytes - s->comm_sent0);
    t8[7] = (double)(s->comm->recv_bytes - s->comm_recv0);
  }
  return TSA_OK;
}

int tsa_session_stats(tsa_session* s, uint64_t* c12, double* ksec) {
  if (!s) return TSA_ERR_ARG;
  if (c12)
    for (int q = 0; q < 12; q++) c12[q] = s->stats[q];
  if (ksec) *ksec = s->kernel_ms / 1e3;
  return TSA_OK;
}

int tsa_resample(void* records, const int32_t* anc, int32_t nchains, uint32_t rec_bytes, void* stream, char* err,
                 size_t errlen) {
  if (!records || !anc || nchains < 1 || rec_bytes == 0 || rec_bytes % 16) {
    set_err(err, errlen, "tsa_resample: need records, anc, nchains >= 1 and rec_bytes a positive multiple of 16");
    return TSA_ERR_ARG;
  }
  for (int c = 0; c < nchains; c++)
    if (anc[c] < 0 || anc[c] >= nchains) {
      set_err(err, errlen, "tsa_resample: ancestor %d of chain %d out of range", anc[c], c);
      return TSA_ERR_ARG;
    }
  cudaStream_t st = (cudaStream_t)stream;
  const size_t bytes = (size_t)nchains * rec_bytes;
  uint8_t* scratch = nullptr;
  int* d_anc = nullptr;
  cudaError_t e = cudaMalloc(&scratch, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&d_anc, nchains * sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_anc, anc, nchains * sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = tsa::launch_copy_chains(static_cast<const uint8_t*>(records), scratch, d_anc, nchains, rec_bytes, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(records, scratch, bytes, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFree(scratch);
  cudaFree(d_anc);
  if (e != cudaSuccess) {
    set_err(err, errlen, "tsa_resample: CUDA error %s", cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? TSA_ERR_NOMEM : TSA_ERR_CUDA;
  }
  return TSA_OK;
}

int tsa_session_info(tsa_session* s, int32_t* v) {
  if (!s || !v) return TSA_ERR_ARG;
  v[0] = s->L.m;
  v[1] = s->L.nint;
  v[2] = s->L.nw;
  v[3] = (int32_t)s->L.rec_bytes;
  v[4] = s->plan.kind == tsa::K_WARP    ? 1
         : s->plan.kind == tsa::K_BLOCK ? (s->plan.cluster == 2 ? 4 : s->plan.gmeta ? 4 + s->plan.gmeta : 2)
                                        : 3;
  v[5] = s->plan.warps_per_cta;
  v[6] = s->plan.grid;
  v[7] = (int32_t)s->plan.smem;
  return TSA_OK;
}

int tsa_session_energies(tsa_session* s, float* lcost, int32_t* sc, int32_t* ns, char* err, size_t errlen) {
  if (!s) return TSA_ERR_ARG;
  if ((int)s->lc.size() != s->nchains) {
    set_err(err, errlen, "no energies yet");
    return TSA_ERR_ARG;
  }
  if (lcost) memcpy(lcost, s->lc.data(), s->nchains * sizeof(float));
  if (sc) memcpy(sc, s->sc.data(), s->nchains * sizeof(int));
  if (ns) memcpy(ns, s->ns.data(), s->nchains * sizeof(int));
  return TSA_OK;
}

int tsa_session_chains(tsa_session* s, uint32_t* trees, uint64_t* labels, char* err, size_t errlen) {
  if (!s) return TSA_ERR_ARG;
  CKR(cudaSetDevice(s->device));
  const Layout& L = s->L;
  std::vector<uint8_t> host((size_t)L.rec_bytes * s->nchains);
  CKR(cudaMemcpyAsync(host.data(), s->d_cur ? s->d_cur : s->d_rec, host.size(), cudaMemcpyDeviceToHost, s->st));
  CKR(cudaStreamSynchronize(s->st));
  for (int c = 0; c < s->nchains; c++) {
    const uint8_t* rec = &host[(size_t)c * L.rec_bytes];
    if (trees) memcpy(trees + (size_t)c * L.nint, rec + L.off_ch, (size_t)L.nint * 4);
    if (labels) memcpy(labels + (size_t)c * L.nint * L.nw, rec, (size_t)L.nint * L.nw * 8);
  }
  return TSA_OK;
}

int tsa_release_cached_memory(void) {
  BlockPool& P = block_pool();
  std::lock_guard<std::mutex> g(P.mu);
  int dev0 = -1;
  cudaGetDevice(&dev0);
  for (auto& kv : P.idle) {
    if (kv.first.kind == 0) cudaSetDevice(kv.first.device);
    raw_free(kv.first.kind, kv.second);
  }
  P.idle.clear();
  P.held[0] = P.held[1] = 0;
  if (dev0 >= 0) cudaSetDevice(dev0);
  return TSA_OK;
}

int tsa_nccl_unique_id(void* id128, char* err, size_t errlen) { return tsa::comm_unique_id(id128, err, errlen); }

int tsa_expf_selftest(int device, uint32_t lo_bits, uint32_t hi_bits, uint64_t* checksum, double* max_rel_fast,
                      char* err, size_t errlen) {
  if (lo_bits < 0x80000000u || hi_bits < lo_bits) {
    set_err(err, errlen, "range must be negative floats with lo <= hi");
    return TSA_ERR_ARG;
  }
  CKR(cudaSetDevice(device));
  unsigned long long* d_sum = nullptr;
  unsigned int* d_err = nullptr;
  CKR(cudaMalloc(&d_sum, sizeof *d_sum));
  CKR(cudaMalloc(&d_err, sizeof *d_err));
  CKR(cudaMemset(d_sum, 0, sizeof *d_sum));
  CKR(cudaMemset(d_err, 0, sizeof *d_err));
  cudaError_t e = tsa::expf_selftest(lo_bits, hi_bits, d_sum, d_err, 0);
  unsigned long long hsum = 0;
  unsigned int herr = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&hsum, d_sum, sizeof hsum, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(&herr, d_err, sizeof herr, cudaMemcpyDeviceToHost);
  cudaFree(d_sum);
  cudaFree(d_err);
  CKR(e);
  float f;
  memcpy(&f, &herr, 4);
  if (checksum) *checksum = hsum;
  if (max_rel_fast) *max_rel_fast = f;
  return TSA_OK;
}

}  // extern "C"
