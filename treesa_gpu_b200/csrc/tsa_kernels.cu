// tsa_kernels.cu -- sm_100a kernels of the B200 TreeSA annealer.
//
// k_anneal_warp<NW, ORDER>: one warp per chain, the chain's whole record staged in shared memory by a
// bulk TMA copy (cp.async.bulk, mbarrier completion) for all sweeps of one beta level, written back by a
// bulk store.  Replaces the reference's k_par (csrc/treesa_gpu.cu:829-997) and k_warp/k_block
// (:585-818) for label sets of up to 512 labels: the whole move is register-resident (NW u64 words per
// set), par-order phases are found by scanning a shrinking list of unvisited nodes instead of all nodes,
// and the per-chain energy (reference k_energy, :1000-1014) is fused into the same launch, read from
// the per-node (cost, size) cache instead of a second pass over the label sets.
//
// k_anneal_block: one CTA per chain for chains too large for shared memory (the 64x64 lattice: 4 MB);
// per-node metadata in shared memory, label sets streamed from HBM with 16-byte loads, G lanes per node.
//
// Every kernel produces bit-identical trees to the reference's CPU port (csrc/cpu_ref.h) for the same
// Philox counters; see tsa_core.h for the arithmetic.
#include <cuda_runtime.h>
#include <stdint.h>

#include "tsa_core.h"
#include "tsa_exp_table.h"
#include "tsa_kernels.cuh"

#define TSA_FIX_QUAL __device__ const
#include "gen/expf_fixups.h"
#undef TSA_FIX_QUAL

namespace tsa {

__constant__ double c_exp_tab[64];

// ------------------------------------------------------------------------------------------------
// PTX helpers: bulk async copies (TMA, non-tensor) with mbarrier completion, bounded waits.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Wait for phase `parity` of the mbarrier, for at most ~2^31 cycles (about a second).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > (1ll << 31)) return false;
  }
}

// ------------------------------------------------------------------------------------------------
// Shared-memory layout of a CTA of k_anneal_warp (computed identically by plan_sweeps)
// ------------------------------------------------------------------------------------------------
__host__ __device__ inline uint32_t rnd_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

struct WarpSmem {
  uint32_t off_bar, off_leaf, off_slots, slot_bytes, off_scr, total;
  int nint2;
  __host__ __device__ static WarpSmem make(const Layout& L, int wpc) {
    WarpSmem w;
    w.nint2 = (int)rnd_up((uint32_t)L.nint, 8);
    w.off_bar = 768;  // [0,256): lse table, [256,768): exp table
    w.off_leaf = rnd_up(w.off_bar + 8u * (uint32_t)wpc, 128);
    w.off_slots = rnd_up(w.off_leaf + (uint32_t)L.m * (uint32_t)L.nw * 8u, 128);
    // record, then pri / par / wl / U (u16 each), then a cz scratch for slice moves
    w.off_scr = L.rec_bytes + 8u * (uint32_t)w.nint2;
    w.slot_bytes = rnd_up(w.off_scr + 4u * (uint32_t)w.nint2, 128);
    w.total = w.off_slots + w.slot_bytes * (uint32_t)wpc;
    return w;
  }
};

// ------------------------------------------------------------------------------------------------
// Label sets in registers
// ------------------------------------------------------------------------------------------------
template <int NW>
struct Set {
  uint64_t w[NW];
};
template <int NW>
__device__ __forceinline__ Set<NW> ldset(const uint64_t* p) {
  Set<NW> s;
  if constexpr (NW % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 2; i++) {
      ulonglong2 t = reinterpret_cast<const ulonglong2*>(p)[i];
      s.w[2 * i] = t.x;
      s.w[2 * i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NW; i++) s.w[i] = p[i];
  }
  return s;
}
template <int NW>
__device__ __forceinline__ void stset(uint64_t* p, const Set<NW>& s) {
  if constexpr (NW % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 2; i++) reinterpret_cast<ulonglong2*>(p)[i] = make_ulonglong2(s.w[2 * i], s.w[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < NW; i++) p[i] = s.w[i];
  }
}

// Per-launch constants kept in registers / shared memory of a warp.
struct WarpCtx {
  int m, nint;
  uint32_t key0, key1;
  float beta, sc_target, sc_weight;
  int slicing;
  const float* lse;      // shared
  const double* exptab;  // shared: 2^(j/64)
  const uint64_t* leaf;  // shared
};

struct Counters {
  unsigned long long prop, acc, steps, visits, sprop, sacc, busy;
};

// One TreeSA proposal at internal node v (one lane).  Semantics: csrc/cpu_ref.h:89-121 (Julia
// optimize_subtree! at one node).  With P the pivot child (left for rules 0,1), O the other child,
// M the pivot's child that moves up and K the one that stays, every rule swaps M and O keeping slots,
// and P gets labels X = (K|O) & (M|D).  Returns v's children word after the move; on accept also
// rewrites P's labels and both (cost, size) words and, for par order, the parents of O and M.
template <int NW, bool PAR>
__device__ __forceinline__ uint32_t visit(const WarpCtx& X_, uint64_t* lab, uint32_t* ch, uint32_t* cz,
                                          const uint64_t* S, uint16_t* par, int v, uint32_t sweep, uint32_t chain,
                                          Counters& cnt) {
  const int m = X_.m;
  const int i = v - m;
  uint32_t chv = ch[i];
  int l = (int)(chv & 0xFFFFu), r = (int)(chv >> 16);
  bool li = l >= m, ri = r >= m;
  if (!li && !ri) return chv;
  U4 rnd = philox10((uint32_t)v, sweep, chain, 0u, X_.key0, X_.key1);
  int rule = pick_rule(li, ri, rnd.x);
  int slotP = rule >> 1;
  int slotM = ((rule ^ (rule >> 1)) & 1) ^ 1;
  int Pn = slotP ? r : l, On = slotP ? l : r;
  uint32_t chp = ch[Pn - m];
  int Mn = slotM ? (int)(chp >> 16) : (int)(chp & 0xFFFFu);
  int Kn = slotM ? (int)(chp & 0xFFFFu) : (int)(chp >> 16);
  const uint64_t* pO = On >= m ? lab + (size_t)(On - m) * NW : X_.leaf + (size_t)On * NW;
  const uint64_t* pK = Kn >= m ? lab + (size_t)(Kn - m) * NW : X_.leaf + (size_t)Kn * NW;
  const uint64_t* pM = Mn >= m ? lab + (size_t)(Mn - m) * NW : X_.leaf + (size_t)Mn * NW;
  Set<NW> D = ldset<NW>(lab + (size_t)i * NW), O = ldset<NW>(pO), K = ldset<NW>(pK), M = ldset<NW>(pM);
  Set<NW> Xs;
  int sx = 0, k2 = 0, k3 = 0;
#pragma unroll
  for (int w = 0; w < NW; w++) {
    uint64_t nm = X_.slicing ? ~S[w] : ~0ull;
    uint64_t x = (K.w[w] | O.w[w]) & (M.w[w] | D.w[w]);
    Xs.w[w] = x;
    uint64_t xm = x & nm;
    sx += __popcll(xm);
    k2 += __popcll(K.w[w] & O.w[w] & ~x & nm);
    k3 += __popcll(xm & M.w[w] & ~D.w[w]);
  }
  uint32_t czv = cz[i], czp = cz[Pn - m];
  int sd = (int)(czv & 0xFFFFu), sp = (int)(czp & 0xFFFFu);
  int cP1 = sx + k2, cV1 = sd + k3;
  float dE = move_energy((int)(czp >> 16), (int)(czv >> 16), sp, sd, sx, cP1, cV1, X_.sc_target, X_.sc_weight, X_.lse);
  cnt.prop++;
  if (metropolis(rnd.y, X_.beta, dE, X_.exptab, kExpfFixX, kExpfFixG, kExpfFixN)) {
    cnt.acc++;
    stset<NW>(lab + (size_t)(Pn - m) * NW, Xs);
    cz[Pn - m] = ((uint32_t)cP1 << 16) | (uint32_t)sx;
    cz[i] = ((uint32_t)cV1 << 16) | (uint32_t)sd;
    uint32_t nchp = slotM ? ((chp & 0xFFFFu) | ((uint32_t)On << 16)) : ((chp & 0xFFFF0000u) | (uint32_t)On);
    uint32_t nchv = slotP ? ((chv & 0xFFFF0000u) | (uint32_t)Mn) : ((chv & 0xFFFFu) | ((uint32_t)Mn << 16));
    ch[Pn - m] = nchp;
    ch[i] = nchv;
    if (PAR) {
      if (On >= m) par[On - m] = (uint16_t)Pn;
      if (Mn >= m) par[Mn - m] = (uint16_t)v;
    }
    chv = nchv;
  }
  return chv;
}

// float log2(2^a + 2^b) with the device's log2f/exp2f, exactly the reference's lse_f (common.h:121-126)
__device__ __forceinline__ float lse_f(float a, float b) {
  float mx = a > b ? a : b;
  float mn = a > b ? b : a;
  if (mx == -INFINITY) return mx;
  return __fadd_rn(mx, log2f(__fadd_rn(1.0f, exp2f(__fsub_rn(mn, mx)))));
}

struct EvalOut {
  float lcost;
  int sc, sc_int, ncand, ns;
};

// Whole-chain energy from the (cost, size) cache, in the reference's lane order (eval_chain,
// csrc/treesa_gpu.cu:386-434): node i accumulated by lane i % 32, then a xor butterfly.
template <int NW>
__device__ EvalOut eval_cached(const WarpCtx& X_, const uint32_t* cz, const uint64_t* S, int leaf_sc, int lane) {
  const unsigned FULL = 0xFFFFFFFFu;
  float acc = -INFINITY;
  int scl = 0, cntl = 0;
  for (int i = lane; i < X_.nint; i += 32) {
    uint32_t w = cz[i];
    int Z = (int)(w & 0xFFFFu);
    acc = lse_f(acc, (float)(int)(w >> 16));
    if (Z > scl) {
      scl = Z;
      cntl = 1;
    } else if (Z == scl) {
      cntl++;
    }
  }
  int scmax = scl;
  for (int o = 16; o > 0; o >>= 1) {
    acc = lse_f(acc, __shfl_xor_sync(FULL, acc, o));
    scmax = max(scmax, __shfl_xor_sync(FULL, scmax, o));
  }
  int cnt = (scl == scmax) ? cntl : 0, ns = 0;
  if (X_.slicing)
    for (int w = lane; w < NW; w += 32) ns += __popcll(S[w]);
  for (int o = 16; o > 0; o >>= 1) {
    cnt += __shfl_xor_sync(FULL, cnt, o);
    ns += __shfl_xor_sync(FULL, ns, o);
  }
  int sc = max(scmax, leaf_sc);
  if (X_.slicing && leaf_sc > scmax) {
    int ll = 0;
    for (int i = lane; i < X_.m; i += 32) {
      int Z = 0;
#pragma unroll
      for (int w = 0; w < NW; w++) Z += __popcll(X_.leaf[(size_t)i * NW + w] & ~S[w]);
      ll = max(ll, Z);
    }
    for (int o = 16; o > 0; o >>= 1) ll = max(ll, __shfl_xor_sync(FULL, ll, o));
    sc = max(scmax, ll);
  }
  return EvalOut{acc, sc, scmax, cnt, ns};
}

// (cost, size) of every internal node on the network sliced by S (lane-strided), into out[].
template <int NW>
__device__ void recompute_cz(const WarpCtx& X_, const uint64_t* lab, const uint32_t* ch, const uint64_t* S,
                             uint32_t* out, int lane) {
  const int m = X_.m;
  for (int i = lane; i < X_.nint; i += 32) {
    uint32_t cw = ch[i];
    int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
    const uint64_t* px = l >= m ? lab + (size_t)(l - m) * NW : X_.leaf + (size_t)l * NW;
    const uint64_t* py = r >= m ? lab + (size_t)(r - m) * NW : X_.leaf + (size_t)r * NW;
    Set<NW> x = ldset<NW>(px), y = ldset<NW>(py), z = ldset<NW>(lab + (size_t)i * NW);
    int Z = 0, K = 0;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      uint64_t nm = ~S[w];
      uint64_t zz = z.w[w] & nm;
      Z += __popcll(zz);
      K += __popcll(x.w[w] & y.w[w] & nm & ~zz);
    }
    out[i] = ((uint32_t)(Z + K) << 16) | (uint32_t)Z;
  }
}

__device__ __forceinline__ float slice_energy(const EvalOut& e, float sc_target, float sc_weight) {
  float pen = (float)e.sc > sc_target ? __fmul_rn(sc_weight, __fsub_rn((float)e.sc, sc_target)) : 0.0f;
  return __fadd_rn(__fadd_rn((float)e.ns, e.lcost), pen);
}

// n-th (0-based) set bit of A & ~S over NW words (S may be null); warp-uniform inputs.
template <int NW>
__device__ __forceinline__ int nth_label(const uint64_t* A, const uint64_t* S, int n) {
  for (int w = 0; w < NW; w++) {
    uint64_t a = A[w] & (S ? ~S[w] : ~0ull);
    int c = __popcll(a);
    if (n < c) {
      for (int k = 0; k < n; k++) a &= a - 1;
      return w * 64 + __ffsll((long long)a) - 1;
    }
    n -= c;
  }
  return -1;
}

// Slice moves of one chain (warp-cooperative): slice_step, csrc/treesa_gpu.cu:445-502.  Costs of the
// proposed slice set are computed into the scratch cache cz2 and committed on accept.
template <int NW>
__device__ void slice_step(const WarpCtx& X_, const SweepArgs& a, uint64_t* lab, uint32_t* ch, uint32_t* cz,
                           uint32_t* cz2, uint64_t* S, uint32_t sweep, uint32_t chain, int lane, Counters& cnt) {
  EvalOut cur = eval_cached<NW>(X_, cz, S, a.leaf_sc, lane);
  float Ecur = slice_energy(cur, X_.sc_target, X_.sc_weight);
  for (int j = 0; j < a.slice_moves; j++) {
    U4 r1 = philox10(0x10000u + 2u * j, sweep, chain, 0u, X_.key0, X_.key1);
    U4 r2 = philox10(0x10001u + 2u * j, sweep, chain, 0u, X_.key0, X_.key1);
    int type;
    if (cur.ns == 0) type = 0;
    else if (cur.ns >= a.max_slices) type = (r1.x >> 31) ? 1 : 2;
    else type = r1.x < 0x80000000u ? 0 : (r1.x < 0xC0000000u ? 1 : 2);
    int ladd = -1, lrem = -1;
    if (type != 1 && cur.ncand > 0 && cur.sc_int > 0) {
      int rr = (int)(r1.y % (uint32_t)cur.ncand), node = -1;
      for (int base = 0; base < X_.nint && node < 0; base += 32) {
        int i = base + lane;
        int Z = i < X_.nint ? (int)(cz[i] & 0xFFFFu) : -1;
        unsigned b = __ballot_sync(0xFFFFFFFFu, Z == cur.sc_int);
        int c = __popc(b);
        if (rr < c) {
          unsigned x = b;
          for (int k = 0; k < rr; k++) x &= x - 1;
          node = base + __ffs(x) - 1;
        } else {
          rr -= c;
        }
      }
      if (node >= 0) ladd = nth_label<NW>(lab + (size_t)node * NW, S, (int)(r1.z % (uint32_t)cur.sc_int));
    }
    if (type != 0) lrem = nth_label<NW>(S, nullptr, (int)(r1.w % (uint32_t)cur.ns));
    if (type == 2 && ladd < 0) type = 1;
    if (type == 0 && ladd < 0) continue;
    __syncwarp();
    if (lane == 0) {
      if (type != 1) S[ladd >> 6] |= 1ull << (ladd & 63);
      if (type != 0) S[lrem >> 6] &= ~(1ull << (lrem & 63));
    }
    __syncwarp();
    recompute_cz<NW>(X_, lab, ch, S, cz2, lane);
    __syncwarp();
    EvalOut nxt = eval_cached<NW>(X_, cz2, S, a.leaf_sc, lane);
    float Enew = slice_energy(nxt, X_.sc_target, X_.sc_weight);
    cnt.sprop++;
    if (metropolis(r2.x, X_.beta, __fsub_rn(Enew, Ecur), X_.exptab, kExpfFixX, kExpfFixG, kExpfFixN)) {
      cnt.sacc++;
      cur = nxt;
      Ecur = Enew;
      for (int i = lane; i < X_.nint; i += 32) cz[i] = cz2[i];
    } else if (lane == 0) {
      if (type != 1) S[ladd >> 6] &= ~(1ull << (ladd & 63));
      if (type != 0) S[lrem >> 6] |= 1ull << (lrem & 63);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------
// k_anneal_warp: nsweeps sweeps of every chain, one warp per chain, chains in shared memory.
// ------------------------------------------------------------------------------------------------
template <int NW, int ORDER>
__global__ void __launch_bounds__(512) k_anneal_warp(SweepArgs a, int wpc) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = a.L;
  const WarpSmem W = WarpSmem::make(L, wpc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* s_lse = reinterpret_cast<float*>(smem);
  double* s_exp = reinterpret_cast<double*>(smem + 256);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + W.off_bar);
  uint64_t* s_leaf = reinterpret_cast<uint64_t*>(smem + W.off_leaf);
  for (int t = threadIdx.x; t < 64; t += blockDim.x) {
    s_lse[t] = a.lse_tab[t];
    s_exp[t] = c_exp_tab[t];
  }
  {
    const int n = L.m * NW;
    for (int t = threadIdx.x; t < n; t += blockDim.x) s_leaf[t] = a.leaf[t];
  }
  if (lane == 0) mbar_init(&s_bar[warp], 1);
  fence_proxy_async();
  __syncthreads();

  WarpCtx X_;
  X_.m = L.m;
  X_.nint = L.nint;
  X_.key0 = a.key0;
  X_.key1 = a.key1;
  X_.beta = a.beta;
  X_.sc_target = a.sc_target;
  X_.sc_weight = a.sc_weight;
  X_.slicing = a.slicing;
  X_.lse = s_lse;
  X_.exptab = s_exp;
  X_.leaf = s_leaf;

  uint8_t* slot = smem + W.off_slots + (size_t)warp * W.slot_bytes;
  uint64_t* lab = reinterpret_cast<uint64_t*>(slot);
  uint32_t* ch = reinterpret_cast<uint32_t*>(slot + L.off_ch);
  uint32_t* cz = reinterpret_cast<uint32_t*>(slot + L.off_cz);
  uint64_t* S = reinterpret_cast<uint64_t*>(slot + L.off_S);
  uint16_t* pri = reinterpret_cast<uint16_t*>(slot + L.rec_bytes);
  uint16_t* par = pri + W.nint2;
  uint16_t* wl = par + W.nint2;
  uint16_t* U = wl + W.nint2;
  uint32_t* cz2 = reinterpret_cast<uint32_t*>(slot + W.off_scr);
  const int m = L.m, nint = L.nint;
  const unsigned FULL = 0xFFFFFFFFu;
  const unsigned lt = (1u << lane) - 1u;
  Counters cnt{};
  uint32_t phase = 0;
  bool failed = false;

  for (int c = blockIdx.x * wpc + warp; c < a.nchains; c += gridDim.x * wpc) {
    uint8_t* grec = a.recs + (size_t)c * L.rec_bytes;
    if (lane == 0) {
      fence_proxy_async();
      mbar_expect_tx(&s_bar[warp], L.rec_bytes);
      bulk_g2s(slot, grec, L.rec_bytes, &s_bar[warp]);
    }
    bool ok = mbar_wait(&s_bar[warp], phase);
    phase ^= 1u;
    if (!__all_sync(FULL, ok)) {
      if (lane == 0) atomicExch(a.err, 1);
      failed = true;
      break;
    }
    __syncwarp();
    const uint32_t chain = (uint32_t)(a.chain0 + c);
    const uint32_t hc = chain_hash(chain, a.key0);
    if (ORDER == 0) {
      for (int i = lane; i < nint; i += 32) {
        uint32_t cw = ch[i];
        int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
        if (l >= m) par[l - m] = (uint16_t)(m + i);
        if (r >= m) par[r - m] = (uint16_t)(m + i);
      }
      if (lane == 0) par[nint - 1] = 0xFFFFu;
      __syncwarp();
    }
    for (int s = 0; s < a.nsweeps; s++) {
      const uint32_t sw = a.sweep0 + (uint32_t)s;
      if (ORDER == 0) {
        // ---- par order: phases of independent sets (cpu_ref.h:133-182, k_par :897-972) ----
        const uint32_t hs = sweep_hash(sw, hc);
        for (int i = lane; i < nint; i += 32) {
          pri[i] = (uint16_t)node_pri((uint32_t)(m + i), hs);
          U[i] = (uint16_t)i;
        }
        int nU = nint;
        __syncwarp();
        for (int guard = 0; guard <= nint; guard++) {
          int nk = 0, nu = 0;
          for (int base = 0; base < nU; base += 32) {
            int j = base + lane;
            bool valid = j < nU;
            int i = valid ? (int)U[j] : 0;
            bool act = false;
            if (valid) {
              uint32_t key = ((uint32_t)pri[i] << 16) | (uint32_t)(m + i);
              act = true;
              int p = par[i];
              if (p != 0xFFFF) {
                uint32_t pp = pri[p - m];
                if (pp && ((pp << 16) | (uint32_t)p) > key) act = false;
              }
              uint32_t cw = ch[i];
              int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
              if (act && l >= m) {
                uint32_t pl = pri[l - m];
                if (pl && ((pl << 16) | (uint32_t)l) > key) act = false;
              }
              if (act && r >= m) {
                uint32_t pr = pri[r - m];
                if (pr && ((pr << 16) | (uint32_t)r) > key) act = false;
              }
            }
            unsigned ba = __ballot_sync(FULL, act), bk = __ballot_sync(FULL, valid && !act);
            __syncwarp();
            if (act) wl[nk + __popc(ba & lt)] = (uint16_t)i;
            if (valid && !act) U[nu + __popc(bk & lt)] = (uint16_t)i;
            nk += __popc(ba);
            nu += __popc(bk);
          }
          nU = nu;
          if (nk == 0) break;
          cnt.steps++;
          __syncwarp();
          for (int j = lane; j < nk; j += 32) {
            int i = wl[j];
            visit<NW, true>(X_, lab, ch, cz, S, par, m + i, sw, chain, cnt);
            pri[i] = 0;
            cnt.visits++;
          }
          cnt.busy += nk;
          __syncwarp();
        }
      } else {
        // ---- pre-order: work list of ready nodes (cpu_ref.h:89-126, k_warp :641-700) ----
        if (lane == 0) wl[0] = (uint16_t)(nint - 1);
        int sp = 1;
        __syncwarp();
        for (int guard = 0; guard <= nint && sp > 0; guard++) {
          int k = min(32, sp), b0 = sp - k;
          int v = lane < k ? m + (int)wl[b0 + lane] : 0;
          __syncwarp();
          uint32_t cw = 0;
          if (lane < k) cw = visit<NW, false>(X_, lab, ch, cz, S, par, v, sw, chain, cnt);
          bool c1 = lane < k && (int)(cw & 0xFFFFu) >= m;
          bool c2 = lane < k && (int)(cw >> 16) >= m;
          unsigned b1 = __ballot_sync(FULL, c1), b2 = __ballot_sync(FULL, c2);
          int pos = b0 + __popc(b1 & lt) + __popc(b2 & lt);
          if (c2) wl[pos++] = (uint16_t)((cw >> 16) - (uint32_t)m);
          if (c1) wl[pos] = (uint16_t)((cw & 0xFFFFu) - (uint32_t)m);
          sp = b0 + __popc(b1) + __popc(b2);
          cnt.steps++;
          cnt.visits += lane < k;
          cnt.busy += k;
          __syncwarp();
        }
      }
      if (a.slice_moves > 0 && (sw + 1) % (uint32_t)a.slice_every == 0) {
        __syncwarp();
        slice_step<NW>(X_, a, lab, ch, cz, cz2, S, sw, chain, lane, cnt);
      }
      __syncwarp();
    }
    // ---- energy of the chain after this launch (fused k_energy) ----
    EvalOut e = eval_cached<NW>(X_, cz, S, a.leaf_sc, lane);
    if (lane == 0) {
      a.out_lc[c] = e.lcost;
      a.out_sc[c] = e.sc;
      a.out_ns[c] = e.ns;
    }
    __syncwarp();
    if (lane == 0) {
      fence_proxy_async();
      bulk_s2g(grec, slot, L.rec_bytes);
      bulk_wait_read();
    }
    __syncwarp();
  }
  if (lane == 0) bulk_wait_all();
  // proposals, accepts and visits are per lane; phases, slice moves and busy lanes are warp-uniform
  unsigned long long v[7] = {cnt.prop, cnt.acc, cnt.steps, cnt.visits, cnt.sprop, cnt.sacc, cnt.busy};
  for (int o = 16; o > 0; o >>= 1) {
    v[0] += __shfl_xor_sync(FULL, v[0], o);
    v[1] += __shfl_xor_sync(FULL, v[1], o);
    v[3] += __shfl_xor_sync(FULL, v[3], o);
  }
  (void)failed;
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < 7; q++)
      if (v[q]) atomicAdd(&a.stats[q], v[q]);
  }
}

// Population resampling: dst chain c <- src chain anc[c] (reference k_copy, :1017-1022).
__global__ void k_copy(const uint4* __restrict__ src, uint4* __restrict__ dst, const int* __restrict__ anc, int n4) {
  const uint4* s = src + (size_t)anc[blockIdx.x] * n4;
  uint4* d = dst + (size_t)blockIdx.x * n4;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d[i] = s[i];
}

// ------------------------------------------------------------------------------------------------
// Host side: plans and launches
// ------------------------------------------------------------------------------------------------
template <int NW, int ORDER>
static cudaError_t launch_warp_t(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  auto k = k_anneal_warp<NW, ORDER>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  k<<<p.grid, 32 * p.warps_per_cta, p.smem, st>>>(a, p.warps_per_cta);
  return cudaGetLastError();
}

template <int ORDER>
static cudaError_t launch_warp_o(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  switch (a.L.nw) {
    case 1: return launch_warp_t<1, ORDER>(a, p, st);
    case 2: return launch_warp_t<2, ORDER>(a, p, st);
    case 4: return launch_warp_t<4, ORDER>(a, p, st);
    case 6: return launch_warp_t<6, ORDER>(a, p, st);
    case 8: return launch_warp_t<8, ORDER>(a, p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t plan_sweeps(const Layout& L, int nchains, int device, LaunchPlan* plan) {
  int nsm = 0, optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) return e;
  bool warp_ok = (L.nw == 1 || L.nw == 2 || L.nw == 4 || L.nw == 6 || L.nw == 8);
  if (warp_ok) {
    // as many chain slots per CTA as fit (at most 16 warps), one CTA per SM
    int wpc = 16;
    while (wpc > 0 && WarpSmem::make(L, wpc).total > (uint32_t)optin) wpc--;
    if (wpc > 0) {
      int need = (nchains + wpc - 1) / wpc;
      // fewer chains than slots: spread them over more CTAs with fewer warps each
      while (wpc > 1 && need < nsm) {
        wpc = (wpc + 1) / 2;
        need = (nchains + wpc - 1) / wpc;
      }
      plan->kind = K_WARP;
      plan->warps_per_cta = wpc;
      plan->grid = need < nsm ? need : nsm;
      plan->smem = WarpSmem::make(L, wpc).total;
      return cudaSuccess;
    }
  }
  return cudaErrorNotSupported;
}

cudaError_t launch_sweeps(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  if (p.kind == K_WARP) return a.order == 0 ? launch_warp_o<0>(a, p, st) : launch_warp_o<1>(a, p, st);
  return cudaErrorNotSupported;
}

cudaError_t launch_copy_chains(const uint8_t* src, uint8_t* dst, const int* anc, int nchains, uint32_t rec_bytes,
                               cudaStream_t st) {
  if (nchains <= 0) return cudaSuccess;
  k_copy<<<nchains, 256, 0, st>>>(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), anc,
                                  (int)(rec_bytes / 16));
  return cudaGetLastError();
}

cudaError_t upload_lse_table(const float* host64, float* dev64, cudaStream_t st) {
  cudaError_t e = cudaMemcpyToSymbolAsync(c_exp_tab, kExp2Tab64, sizeof(kExp2Tab64), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaMemcpyAsync(dev64, host64, 64 * sizeof(float), cudaMemcpyHostToDevice, st);
}

int fixup_count() { return kExpfFixN; }

}  // namespace tsa
