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
// ORDER 0 is par order, 1 pre-order, 2 par order with the --par-band / --par-follow variants (its own
// instantiation, so that plain par order keeps its registers).
//
// k_anneal_block: one CTA per chain for chains too large for shared memory; per-node metadata in shared
// memory, label sets streamed from HBM in 16-byte chunks: par phases with chunk summaries as flat
// (node, chunk) item lists spread over all threads (par_phase_flat), otherwise G lanes per node.
//
// k_anneal_cluster: par order with chunk summaries when chains are fewer than half the SMs (the 64x64
// lattice: 72 chains of 4 MB): a cluster of two CTAs per chain, metadata replicated in both CTAs'
// shared memory and kept equal by distributed-shared-memory stores; per phase the CTAs meet at a split
// cluster barrier (arrive after the scan, wait before the first store into the other copy) and at a full
// one at its end.
//
// Every kernel produces bit-identical trees to the reference's CPU port (csrc/cpu_ref.h) for the same
// Philox counters; see tsa_core.h for the arithmetic.
#include <cooperative_groups.h>
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

// Wait for phase `parity` of the mbarrier, for at most `limit` SM cycles (2^31 by default: about a second).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > limit) return false;
  }
}

// ------------------------------------------------------------------------------------------------
// Shared-memory layout of a CTA of k_anneal_warp (computed identically by plan_sweeps)
// ------------------------------------------------------------------------------------------------
__host__ __device__ inline uint32_t rnd_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

struct WarpSmem {
  uint32_t off_bar, off_leaf, off_slots, slot_bytes, off_par, off_scr, total;
  int nint2, nkey;
  __host__ __device__ static WarpSmem make(const Layout& L, int wpc, int slice_moves) {
    WarpSmem w;
    w.nint2 = (int)rnd_up((uint32_t)L.nint, 8);
    w.nkey = (int)rnd_up((uint32_t)L.nint + 1u, 4);  // par-order keys + a zero sentinel at [nint]
    w.off_bar = 768;  // [0,256): lse table, [256,768): exp table
    w.off_leaf = rnd_up(w.off_bar + 8u * (uint32_t)wpc, 128);
    w.off_slots = rnd_up(w.off_leaf + (uint32_t)L.m * (uint32_t)L.nw * 8u, 128);
    // record, then key (u32), par / wl / U (u16 each), then a cz scratch for slice moves
    w.off_par = L.rec_bytes + 4u * (uint32_t)w.nkey;
    w.off_scr = w.off_par + 6u * (uint32_t)w.nint2;
    w.slot_bytes = rnd_up(w.off_scr + (slice_moves > 0 ? 4u * (uint32_t)w.nint2 : 0u), 128);
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

// The same loads and stores through 32-bit shared-memory addresses (the warp kernels keep the chain and
// the leaf table in shared memory): one select and one multiply-add a set instead of 64-bit pointers.
// The memory clobber keeps them in order with the kernels' other shared-memory accesses.
__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
template <int NW>
__device__ __forceinline__ Set<NW> ldset_s(uint32_t a) {
  Set<NW> s;
  if constexpr (NW % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 2; i++)
      asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(s.w[2 * i]), "=l"(s.w[2 * i + 1]) : "r"(a + 16u * i) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < NW; i++) asm volatile("ld.shared.u64 %0, [%1];" : "=l"(s.w[i]) : "r"(a + 8u * i) : "memory");
  }
  return s;
}
template <int NW>
__device__ __forceinline__ void stset_s(uint32_t a, const Set<NW>& s) {
  if constexpr (NW % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NW / 2; i++)
      asm volatile("st.shared.v2.u64 [%0], {%1, %2};" ::"r"(a + 16u * i), "l"(s.w[2 * i]), "l"(s.w[2 * i + 1]) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < NW; i++) asm volatile("st.shared.u64 [%0], %1;" ::"r"(a + 8u * i), "l"(s.w[i]) : "memory");
  }
}

// Per-launch constants kept in registers / shared memory of a warp.
struct WarpCtx {
  int m, nint;
  uint32_t key0, key1;
  float beta, sc_target, sc_weight;
  int slicing;
  int exp_device;
  int mode;  // energy mode of the launch (the model kernels: 1 gpu, 2 h100)
  ModelParams mp;
  const float* lse;      // shared
  const double* exptab;  // shared: 2^(j/64)
  const uint64_t* leaf;  // shared
  // pre-order: the sweep's random numbers of every node, drawn up front (see k_anneal_warp), word i for
  // node m + i: bits 8..31 of Philox .y (all the Metropolis test reads) | the top two bits of .x (all
  // the rule pick reads)
  const uint32_t* rtab;
};

struct Counters {
  unsigned long long prop, acc, steps, visits, sprop, sacc, busy, chunks, chunks_acc;
};
// per-chain counts of one lane (32-bit adds in the inner loops), added into Counters after each chain
struct ChainCounters {
  uint32_t prop, acc, steps, visits, sprop, sacc, busy;
  __device__ __forceinline__ void flush(Counters& c) {
    c.prop += prop;
    c.acc += acc;
    c.steps += steps;
    c.visits += visits;
    c.sprop += sprop;
    c.sacc += sacc;
    c.busy += busy;
    *this = ChainCounters{};
  }
};
// per-chain counts of one thread of the CTA kernels (32 bits: a thread's share of one chain), added into
// the launch's device counters at the end of every chain, so that no 64-bit totals stay live in registers
struct BlkCounters {
  uint32_t prop, acc, steps, visits, sprop, sacc, busy, chunks, chunks_acc;
  // every thread: its own proposals/accepts/visits/items; steps counted by one thread; slice moves by all
  // 32 lanes of warp 0 (slice_div 32), or by two CTAs of which one reports (slice_div 0 in the other)
  __device__ __forceinline__ void flush(unsigned long long* stats, int slice_div) {
    uint32_t v[9] = {prop, acc, steps, visits, sprop, sacc, busy, chunks, chunks_acc};
#pragma unroll
    for (int q = 0; q < 9; q++) v[q] = __reduce_add_sync(0xFFFFFFFFu, v[q]);
    if ((threadIdx.x & 31) == 0) {
      v[4] = slice_div ? v[4] / (uint32_t)slice_div : 0u;
      v[5] = slice_div ? v[5] / (uint32_t)slice_div : 0u;
      const int slot[9] = {0, 1, 2, 3, 4, 5, 6, 8, 9};
#pragma unroll
      for (int q = 0; q < 9; q++)
        if (v[q]) atomicAdd(&stats[slot[q]], (unsigned long long)v[q]);
    }
    *this = BlkCounters{};
  }
};

// Metropolis: host-libm-exact (default) or with the device's expf as the reference's GPU binary
__device__ __forceinline__ bool accept_rt(int exp_device, float beta, const double* exptab, uint32_t r, float dE) {
  if (exp_device) {
    float u = (float)(r >> 8) * (1.0f / 16777216.0f);
    return u < expf(__fmul_rn(-beta, dE));
  }
  return metropolis(r, beta, dE, exptab, kExpfFixX, kExpfFixG, kExpfFixN);
}
__device__ __forceinline__ bool accept(const WarpCtx& X_, uint32_t r, float dE) {
  return accept_rt(X_.exp_device, X_.beta, X_.exptab, r, dE);
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

// ------------------------------------------------------------------------------------------------
// Energy modes gpu / h100 (csrc/common.h:128-162): log2 of the modeled time of one pairwise
// contraction (x, y) -> z with label counts B = |x&y&z|, M = |x&~y&z|, N = |~x&y&z|, K = |x&y&~z|,
// in the device's float arithmetic (log2f / exp2f through lse_f), as the reference's kernels.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float gpu_lt(int B, int M, int N, int K, const ModelParams& P) {
  const int Me = M > P.m0 ? M : P.m0, Ne = N > P.n0 ? N : P.n0, Ke = K > P.k0 ? K : P.k0;
  const float lops = __fsub_rn((float)(1 + B + Me + Ne + Ke), P.lpeak);
  const float lbits = __fsub_rn(lse_f(lse_f((float)(B + M + K), (float)(B + N + K)), (float)(B + M + N)), P.lbw);
  return lse_f(lops > lbits ? lops : lbits, P.llaunch);
}
__device__ __forceinline__ float h100_lt(int B, int M, int N, int K, const ModelParams& P) {
  if (B + M + N <= P.small_rank) return __fadd_rn(P.lsmall_cell, (float)(B + M + N + K));
  const float la = (float)(B + M + K), lb = (float)(B + N + K), lc = (float)(B + M + N);
  const float lab = lse_f(la, lb), lmoved = lse_f(lab, lc);
  const float perm = __fadd_rn(P.lperm2, lab);
  float best = lse_f(__fadd_rn(P.lcc_bit, lmoved), __fadd_rn(P.lcc_cell, (float)(B + M + N + K)));
  const int MN = M > N ? M : N;
  if (K >= 7 && MN >= 5) {
    const int Me = M > 6 ? M : 6, Ne = N > 6 ? N : 6, Ke = K > 8 ? K : 8;
    const float tc = lse_f(lse_f(__fadd_rn(P.ltc_bit, lmoved), __fadd_rn(P.ltc_pad, (float)(B + Me + Ne + Ke))),
                           __fadd_rn(P.ltc_out, lc));
    best = tc < best ? tc : best;
  }
  return lse_f(lse_f(P.l3launch, perm), best);
}
__device__ __forceinline__ float model_cost(int mode, const ModelParams& P, int B, int M, int N, int K) {
  return mode == 1 ? gpu_lt(B, M, N, K, P) : h100_lt(B, M, N, K, P);
}
// label counts of (x, y) -> z on one masked word (count3, common.h:172-177)
struct C4 {
  int B, M, N, K;
};
__device__ __forceinline__ void count3(uint64_t x, uint64_t y, uint64_t z, C4& c) {
  c.B += __popcll(x & y & z);
  c.M += __popcll(x & ~y & z);
  c.N += __popcll(~x & y & z);
  c.K += __popcll(x & y & ~z);
}
// dE of a move from the costs of the contractions before (t0) and after (t1) and the sizes
// (energy_from_counts, common.h:198-222)
__device__ __forceinline__ float model_energy(float t0, float t1, int sp, int sd, int sx, float sc_target,
                                              float sc_weight) {
  const int sc0 = sp > sd ? sp : sd, sc1 = sx > sd ? sx : sd, dsc = sc1 - sc0, scmax = sc0 > sc1 ? sc0 : sc1;
  const float w = ((float)scmax > sc_target) ? sc_weight : 0.0f;
  return __fadd_rn(__fmul_rn(w, (float)dsc), __fsub_rn(t1, t0));
}

// One TreeSA proposal at internal node v (one lane).  Semantics: csrc/cpu_ref.h:89-121 (Julia
// optimize_subtree! at one node).  With P the pivot child (left for rules 0,1), O the other child,
// M the pivot's child that moves up and K the one that stays, every rule swaps M and O keeping slots,
// and P gets labels X = (K|O) & (M|D).  propose() only reads; apply() rewrites P's labels, both
// (cost, size) words, both children words and, for par order, the parents of O and M.  A lane may
// evaluate two nodes of one par phase before it writes either: within a phase the reads of one
// proposal and the writes of another never touch the same word (the nodes are pairwise non-adjacent,
// and a move at v writes only v, its pivot child and the parents of O and M).
// NM holds the labels that are not sliced (all ones without slicing).
template <int NW>
struct Prop {
  Set<NW> X;
  uint32_t nchv, nchp;
  int i, Pn, On, Mn, cP1, sx, cV1, sd;
  bool acc;
};
// MODEL: energy modes gpu / h100; the four contractions (K,M)->P, (P,O)->D, (K,O)->X, (X,M)->D are
// counted from the label sets as the reference does (cpu_ref.h:69-72), which also needs P's set.
// PRE: the node's random numbers come from X_.rtab instead of a Philox call on the move's critical path.
template <int NW, bool MODEL = false, bool PRE = false>
__device__ __forceinline__ Prop<NW> propose(const WarpCtx& X_, const uint64_t* lab, const uint32_t* ch,
                                            const uint32_t* cz, const Set<NW>& NM, int v, uint32_t chv,
                                            uint32_t sweep, uint32_t chain) {
  const int m = X_.m;
  Prop<NW> p;
  p.i = v - m;
  int l = (int)(chv & 0xFFFFu), r = (int)(chv >> 16);
  bool li = l >= m, ri = r >= m;
  U4 rnd;
  if constexpr (PRE) {
    const uint32_t pk = X_.rtab[v - m];
    rnd.x = pk << 30;
    rnd.y = pk & 0xFFFFFF00u;
  } else {
    rnd = philox10((uint32_t)v, sweep, chain, 0u, X_.key0, X_.key1);
  }
  int rule = pick_rule(li, ri, rnd.x);
  int slotP = rule >> 1;
  int slotM = ((rule ^ (rule >> 1)) & 1) ^ 1;
  p.Pn = slotP ? r : l;
  p.On = slotP ? l : r;
  uint32_t chp = ch[p.Pn - m];
  p.Mn = slotM ? (int)(chp >> 16) : (int)(chp & 0xFFFFu);
  int Kn = slotM ? (int)(chp & 0xFFFFu) : (int)(chp >> 16);
  // node n's set: internal at labA + n * 8NW (wrapping arithmetic), leaf at leafA + n * 8NW
  const uint32_t labA = saddr(lab) - (uint32_t)(m * NW * 8), leafA = saddr(X_.leaf);
  auto sa = [&](int n) { return (n >= m ? labA : leafA) + (uint32_t)n * (uint32_t)(NW * 8); };
  Set<NW> D = ldset_s<NW>(labA + (uint32_t)v * (uint32_t)(NW * 8)), O = ldset_s<NW>(sa(p.On)),
          K = ldset_s<NW>(sa(Kn)), M = ldset_s<NW>(sa(p.Mn));
  int sx = 0, k2 = 0, k3 = 0;
  C4 c[4] = {};
#pragma unroll
  for (int w = 0; w < NW; w++) {
    uint64_t x = (K.w[w] | O.w[w]) & (M.w[w] | D.w[w]);
    p.X.w[w] = x;
    uint64_t xm = x & NM.w[w];
    sx += __popcll(xm);
    k2 += __popcll(K.w[w] & O.w[w] & ~x & NM.w[w]);
    k3 += __popcll(xm & M.w[w] & ~D.w[w]);
  }
  if constexpr (MODEL) {
    const Set<NW> Pset = ldset_s<NW>(labA + (uint32_t)p.Pn * (uint32_t)(NW * 8));
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const uint64_t nm = NM.w[w], k = K.w[w] & nm, mm = M.w[w] & nm, pp = Pset.w[w] & nm, o = O.w[w] & nm,
                     d = D.w[w] & nm, x = p.X.w[w] & nm;
      count3(k, mm, pp, c[0]);
      count3(pp, o, d, c[1]);
      count3(k, o, x, c[2]);
      count3(x, mm, d, c[3]);
    }
  }
  uint32_t czv = cz[p.i], czp = cz[p.Pn - m];
  p.sd = (int)(czv & 0xFFFFu);
  int sp = (int)(czp & 0xFFFFu);
  p.sx = sx;
  p.cP1 = sx + k2;
  p.cV1 = p.sd + k3;
  float dE;
  if constexpr (MODEL) {
    auto cost = [&](const C4& q) { return model_cost(X_.mode, X_.mp, q.B, q.M, q.N, q.K); };
    dE = model_energy(lse_f(cost(c[0]), cost(c[1])), lse_f(cost(c[2]), cost(c[3])), sp, p.sd, sx, X_.sc_target,
                      X_.sc_weight);
  } else {
    dE = move_energy((int)(czp >> 16), (int)(czv >> 16), sp, p.sd, sx, p.cP1, p.cV1, X_.sc_target, X_.sc_weight,
                     X_.lse);
  }
  p.acc = accept(X_, rnd.y, dE);
  p.nchp = slotM ? ((chp & 0xFFFFu) | ((uint32_t)p.On << 16)) : ((chp & 0xFFFF0000u) | (uint32_t)p.On);
  p.nchv = slotP ? ((chv & 0xFFFF0000u) | (uint32_t)p.Mn) : ((chv & 0xFFFFu) | ((uint32_t)p.Mn << 16));
  return p;
}
template <int NW, bool PAR>
__device__ __forceinline__ void apply(const Prop<NW>& p, int m, uint64_t* lab, uint32_t* ch, uint32_t* cz,
                                      uint16_t* par) {
  stset_s<NW>(saddr(lab) + (uint32_t)(p.Pn - m) * (uint32_t)(NW * 8), p.X);
  cz[p.Pn - m] = ((uint32_t)p.cP1 << 16) | (uint32_t)p.sx;
  cz[p.i] = ((uint32_t)p.cV1 << 16) | (uint32_t)p.sd;
  ch[p.Pn - m] = p.nchp;
  ch[p.i] = p.nchv;
  if (PAR) {
    if (p.On >= m) par[p.On - m] = (uint16_t)p.Pn;
    if (p.Mn >= m) par[p.Mn - m] = (uint16_t)(m + p.i);
  }
}
// propose + apply at one node; returns v's children word after the move (unchanged for a leaf-only node)
template <int NW, bool PAR, typename C, bool MODEL = false, bool PRE = false>
__device__ __forceinline__ uint32_t visit(const WarpCtx& X_, uint64_t* lab, uint32_t* ch, uint32_t* cz,
                                          const Set<NW>& NM, uint16_t* par, int v, uint32_t sweep, uint32_t chain,
                                          C& cnt) {
  const uint32_t chv = ch[v - X_.m];
  if ((int)(chv & 0xFFFFu) < X_.m && (int)(chv >> 16) < X_.m) return chv;
  Prop<NW> p = propose<NW, MODEL, PRE>(X_, lab, ch, cz, NM, v, chv, sweep, chain);
  cnt.prop++;
  if (p.acc) {
    cnt.acc++;
    apply<NW, PAR>(p, X_.m, lab, ch, cz, par);
    return p.nchv;
  }
  return chv;
}

// Not-sliced label mask of a chain in registers
template <int NW>
__device__ __forceinline__ Set<NW> not_sliced(const uint64_t* S, int slicing) {
  Set<NW> nm;
#pragma unroll
  for (int w = 0; w < NW; w++) nm.w[w] = slicing ? ~S[w] : ~0ull;
  return nm;
}


// Whole-chain energy in the reference's lane order (eval_chain, csrc/treesa_gpu.cu:386-434): node i
// accumulated by lane i % 32, then a xor butterfly.  node(i, Z) returns node i's log2 cost and sets its
// size Z.
template <int NW, typename F>
__device__ EvalOut eval_nodes(const WarpCtx& X_, const uint64_t* S, int leaf_sc, int lane, F&& node) {
  const unsigned FULL = 0xFFFFFFFFu;
  float acc = -INFINITY;
  int scl = 0, cntl = 0;
  for (int i = lane; i < X_.nint; i += 32) {
    int Z;
    const float cost = node(i, Z);
    acc = lse_f(acc, cost);
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
// tc: from the (cost, size) cache
template <int NW>
__device__ EvalOut eval_cached(const WarpCtx& X_, const uint32_t* cz, const uint64_t* S, int leaf_sc, int lane) {
  return eval_nodes<NW>(X_, S, leaf_sc, lane, [&](int i, int& Z) {
    const uint32_t w = cz[i];
    Z = (int)(w & 0xFFFFu);
    return (float)(int)(w >> 16);
  });
}
// the gpu / h100 models: each node's contraction counted from the label sets (sliced by S)
template <int NW>
__device__ EvalOut eval_model(const WarpCtx& X_, const uint64_t* lab, const uint32_t* ch, const uint64_t* S,
                              int leaf_sc, int lane) {
  const int m = X_.m;
  return eval_nodes<NW>(X_, S, leaf_sc, lane, [&](int i, int& Z) {
    const uint32_t cw = ch[i];
    const int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
    const Set<NW> x = ldset<NW>(l >= m ? lab + (size_t)(l - m) * NW : X_.leaf + (size_t)l * NW);
    const Set<NW> y = ldset<NW>(r >= m ? lab + (size_t)(r - m) * NW : X_.leaf + (size_t)r * NW);
    const Set<NW> z = ldset<NW>(lab + (size_t)i * NW);
    C4 c{};
    Z = 0;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const uint64_t nm = X_.slicing ? ~S[w] : ~0ull, zz = z.w[w] & nm;
      count3(x.w[w] & nm, y.w[w] & nm, zz, c);
      Z += __popcll(zz);
    }
    return model_cost(X_.mode, X_.mp, c.B, c.M, c.N, c.K);
  });
}
template <int NW, bool MODEL>
__device__ __forceinline__ EvalOut eval_w(const WarpCtx& X_, const uint64_t* lab, const uint32_t* ch,
                                          const uint32_t* cz, const uint64_t* S, int leaf_sc, int lane) {
  if constexpr (MODEL) return eval_model<NW>(X_, lab, ch, S, leaf_sc, lane);
  else return eval_cached<NW>(X_, cz, S, leaf_sc, lane);
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
template <int NW, typename C, bool MODEL = false>
__device__ void slice_step(const WarpCtx& X_, const SweepArgs& a, uint64_t* lab, uint32_t* ch, uint32_t* cz,
                           uint32_t* cz2, uint64_t* S, uint32_t sweep, uint32_t chain, int lane, C& cnt) {
  EvalOut cur = eval_w<NW, MODEL>(X_, lab, ch, cz, S, a.leaf_sc, lane);
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
    EvalOut nxt = eval_w<NW, MODEL>(X_, lab, ch, cz2, S, a.leaf_sc, lane);
    float Enew = slice_energy(nxt, X_.sc_target, X_.sc_weight);
    cnt.sprop++;
    if (accept(X_, r2.x, __fsub_rn(Enew, Ecur))) {
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
// Depth of every internal node (root 0) by pointer jumping: word i = depth << 16 | ancestor (0xFFFF once
// the root is reached); every round adds the ancestor's depth and jumps to the ancestor's ancestor, so
// log2(depth) + 1 rounds suffice.  Two buffers of nint words; the result ends in A.  One warp.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void warp_depths(const uint16_t* par, int m, int nint, uint32_t*& A, uint32_t*& Bq,
                                            int lane) {
  for (int i = lane; i < nint; i += 32) {
    const int p = par[i];
    A[i] = p == 0xFFFF ? 0xFFFFu : ((1u << 16) | (uint32_t)(p - m));
  }
  __syncwarp();
  for (int r = 0; r < 18; r++) {
    bool more = false;
    for (int i = lane; i < nint; i += 32) {
      uint32_t x = A[i];
      const uint32_t an = x & 0xFFFFu;
      if (an < (uint32_t)nint) {  // 0xFFFF: the root is reached
        const uint32_t y = A[an];
        x = (((x >> 16) + (y >> 16)) << 16) | (y & 0xFFFFu);
        more |= (y & 0xFFFFu) != 0xFFFFu;
      }
      Bq[i] = x;
    }
    __syncwarp();
    uint32_t* t = A;
    A = Bq;
    Bq = t;
    if (!__any_sync(0xFFFFFFFFu, more)) break;
  }
}

// The same over a CTA; the result ends in the buffer U32 (which the caller then reads while it
// overwrites the other one).
__device__ __forceinline__ void block_depths(const uint16_t* par, int m, int nint, uint32_t* A0, uint32_t* U32) {
  const int tid = threadIdx.x, T = blockDim.x;
  uint32_t *A = A0, *Bq = U32;
  for (int i = tid; i < nint; i += T) {
    const int p = par[i];
    A[i] = p == 0xFFFF ? 0xFFFFu : ((1u << 16) | (uint32_t)(p - m));
  }
  __syncthreads();
  for (int r = 0; r < 18; r++) {
    bool more = false;
    for (int i = tid; i < nint; i += T) {
      uint32_t x = A[i];
      const uint32_t an = x & 0xFFFFu;
      if (an < (uint32_t)nint) {  // 0xFFFF: the root is reached
        const uint32_t y = A[an];
        x = (((x >> 16) + (y >> 16)) << 16) | (y & 0xFFFFu);
        more |= (y & 0xFFFFu) != 0xFFFFu;
      }
      Bq[i] = x;
    }
    uint32_t* t = A;
    A = Bq;
    Bq = t;
    if (!__syncthreads_or(more)) break;
  }
  if (A != U32) {
    for (int i = tid; i < nint; i += T) U32[i] = A[i];
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// k_anneal_warp: nsweeps sweeps of every chain, one warp per chain, chains in shared memory.
// ------------------------------------------------------------------------------------------------
template <int NW, int ORDER, bool MODEL>
__global__ void __launch_bounds__(512) k_anneal_warp(SweepArgs a, int wpc) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = a.L;
  const WarpSmem W = WarpSmem::make(L, wpc, a.slice_moves);
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
  X_.exp_device = a.exp_device;
  X_.mode = a.mode;
  X_.mp = a.mp;
  X_.lse = s_lse;
  X_.exptab = s_exp;
  X_.leaf = s_leaf;
  X_.rtab = nullptr;

  uint8_t* slot = smem + W.off_slots + (size_t)warp * W.slot_bytes;
  uint64_t* lab = reinterpret_cast<uint64_t*>(slot);
  uint32_t* ch = reinterpret_cast<uint32_t*>(slot + L.off_ch);
  uint32_t* cz = reinterpret_cast<uint32_t*>(slot + L.off_cz);
  uint64_t* S = reinterpret_cast<uint64_t*>(slot + L.off_S);
  uint32_t* key = reinterpret_cast<uint32_t*>(slot + L.rec_bytes);
  uint16_t* par = reinterpret_cast<uint16_t*>(slot + W.off_par);
  uint16_t* wl = par + W.nint2;
  uint16_t* U = wl + W.nint2;
  uint32_t* cz2 = reinterpret_cast<uint32_t*>(slot + W.off_scr);
  const int m = L.m, nint = L.nint, nint2 = W.nint2;
  const unsigned FULL = 0xFFFFFFFFu;
  const unsigned lt = (1u << lane) - 1u;
  Counters tot{};
  ChainCounters cnt{};
  uint32_t phase = 0;
  bool failed = false;

  for (int c = blockIdx.x * wpc + warp; c < a.nchains; c += gridDim.x * wpc) {
    uint8_t* grec = a.recs + (size_t)c * L.rec_bytes;
    if (lane == 0) {
      fence_proxy_async();
      mbar_expect_tx(&s_bar[warp], L.rec_bytes);
      if (!a.debug_arm_only) bulk_g2s(slot, grec, L.rec_bytes, &s_bar[warp]);
    }
    bool ok = mbar_wait(&s_bar[warp], phase, a.wait_cycles);
    phase ^= 1u;
    if (!__all_sync(FULL, ok)) {
      if (lane == 0) atomicExch(a.err, 1);
      failed = true;
      break;
    }
    __syncwarp();
    const uint32_t chain = (uint32_t)(a.chain0 + c);
    const uint32_t hc = chain_hash(chain, a.key0);
    if (ORDER != 1) {
      for (int i = lane; i < nint; i += 32) {
        uint32_t cw = ch[i];
        int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
        if (l >= m) par[l - m] = (uint16_t)(m + i);
        if (r >= m) par[r - m] = (uint16_t)(m + i);
      }
      if (lane == 0) par[nint - 1] = 0xFFFFu;
      __syncwarp();
    }
    Set<NW> NM = not_sliced<NW>(S, X_.slicing);
    for (int s = 0; s < a.nsweeps; s++) {
      const uint32_t sw = a.sweep0 + (uint32_t)s;
      if (ORDER != 1) {
        // ---- par order: phases of independent sets (cpu_ref.h:133-182, k_par :897-972) ----
        // key[i] = priority << 16 | node id while node m+i is unvisited, 0 once visited; key[nint] = 0 is
        // the sentinel read for a leaf child or the root's parent, so a node is active iff its key
        // exceeds the keys of its parent and children.
        const uint32_t hs = sweep_hash(sw, hc);
        if (ORDER == 2 && a.par_band > 0) {
          // depth of every node at the start of the sweep, by pointer jumping over two buffers that are
          // free until the priorities are set: key[] and the wl/U lists (read as u32)
          uint32_t* A = key;
          uint32_t* Bq = reinterpret_cast<uint32_t*>(wl);
          warp_depths(par, m, nint, A, Bq, lane);
          // A now holds depth << 16 (| 0xFFFF): each lane reads and rewrites only its own nodes' words
          for (int i = lane; i < nint; i += 32)
            key[i] = (band_pri(node_pri((uint32_t)(m + i), hs), (int)(A[i] >> 16), a.par_band) << 16) |
                     (uint32_t)(m + i);
          __syncwarp();
          for (int i = lane; i < nint; i += 32) U[i] = (uint16_t)i;
        } else {
          for (int i = lane; i < nint; i += 32) {
            key[i] = (node_pri((uint32_t)(m + i), hs) << 16) | (uint32_t)(m + i);
            U[i] = (uint16_t)i;
          }
        }
        if (lane == 0) key[nint] = 0u;
        int nU = nint;
        __syncwarp();
        // par_follow: an accepted first visit (odd priority) re-arms its pivot child P with an even
        // priority if the sweep already visited it; P goes back on the unvisited list, and its second
        // visit draws Philox with the sweep's top bit set (cpu_ref.h:168-175)
        const bool follow = ORDER == 2 && a.par_follow != 0;
        auto swv = [&](uint32_t k) { return ((k >> 16) & 1u) ? sw : follow_sweep(sw); };
        auto rearm = [&](const Prop<NW>& p, uint32_t k) -> int {
          if (!follow || !p.acc || !((k >> 16) & 1u)) return -1;
          const int pi = p.Pn - m;
          if (key[pi] != 0u) return -1;
          key[pi] = (follow_pri((uint32_t)p.Pn, hs) << 16) | (uint32_t)p.Pn;
          return pi;
        };
        auto push = [&](int r0, int r1) {  // re-armed nodes onto the unvisited list (all lanes)
          const unsigned b0 = __ballot_sync(FULL, r0 >= 0), b1 = __ballot_sync(FULL, r1 >= 0);
          if (r0 >= 0) U[nU + __popc(b0 & lt)] = (uint16_t)r0;
          if (r1 >= 0) U[nU + __popc(b0) + __popc(b1 & lt)] = (uint16_t)r1;
          nU += __popc(b0) + __popc(b1);
        };
        const int max_phases = follow ? 2 * nint : nint;
        for (int guard = 0; guard <= max_phases; guard++) {
          int nk = 0, nu = 0, nc = 0;
          // two list entries per lane per step: their shared-memory loads overlap
          for (int base = 0; base < nU; base += 64) {
            const int j0 = base + lane, j1 = base + 32 + lane;
            const bool v0 = j0 < nU, v1 = j1 < nU;
            const int i0 = v0 ? (int)U[j0] : nint, i1 = v1 ? (int)U[j1] : nint;
            const uint32_t k0 = key[i0], k1 = key[i1];
            const uint32_t c0 = ch[v0 ? i0 : 0], c1 = ch[v1 ? i1 : 0];
            const int p0 = par[v0 ? i0 : 0], p1 = par[v1 ? i1 : 0];
            auto idx = [&](int n) { return n >= m ? n - m : nint; };
            const int l0 = (int)(c0 & 0xFFFFu), r0 = (int)(c0 >> 16), l1 = (int)(c1 & 0xFFFFu), r1 = (int)(c1 >> 16);
            const uint32_t q0 = max(key[p0 == 0xFFFF ? nint : p0 - m], max(key[idx(l0)], key[idx(r0)]));
            const uint32_t q1 = max(key[p1 == 0xFFFF ? nint : p1 - m], max(key[idx(l1)], key[idx(r1)]));
            const bool a0 = v0 && k0 > q0, a1 = v1 && k1 > q1;
            const bool ch0 = a0 && l0 < m && r0 < m, ch1 = a1 && l1 < m && r1 < m;
            const bool pr0 = a0 && !ch0, pr1 = a1 && !ch1;
            const bool kp0 = v0 && !a0, kp1 = v1 && !a1;
            const unsigned bp0 = __ballot_sync(FULL, pr0), bp1 = __ballot_sync(FULL, pr1);
            const unsigned bc0 = __ballot_sync(FULL, ch0), bc1 = __ballot_sync(FULL, ch1);
            const unsigned bk0 = __ballot_sync(FULL, kp0), bk1 = __ballot_sync(FULL, kp1);
            __syncwarp();
            if (pr0) wl[nk + __popc(bp0 & lt)] = (uint16_t)i0;
            if (pr1) wl[nk + __popc(bp0) + __popc(bp1 & lt)] = (uint16_t)i1;
            if (ch0) wl[nint2 - 1 - (nc + __popc(bc0 & lt))] = (uint16_t)i0;
            if (ch1) wl[nint2 - 1 - (nc + __popc(bc0) + __popc(bc1 & lt))] = (uint16_t)i1;
            if (kp0) U[nu + __popc(bk0 & lt)] = (uint16_t)i0;
            if (kp1) U[nu + __popc(bk0) + __popc(bk1 & lt)] = (uint16_t)i1;
            nk += __popc(bp0) + __popc(bp1);
            nc += __popc(bc0) + __popc(bc1);
            nu += __popc(bk0) + __popc(bk1);
          }
          nU = nu;
          if (nk + nc == 0) break;
          cnt.steps++;
          __syncwarp();
          // active nodes whose children are both leaves make no proposal: they only become visited
          for (int j = lane; j < nc; j += 32) {
            key[wl[nint2 - 1 - j]] = 0u;
            cnt.visits++;
          }
          // more than 32 proposals: two per lane, both evaluated before either is applied (tc mode and sets
          // of up to 4 words: above that the two proposals no longer fit in registers)
          int j = lane;
          constexpr bool TWO = !MODEL && NW <= 4;
          for (; TWO && nk - (j - lane) > 32; j += 64) {
            const int ja = j, jb = j + 32;
            const bool vb = jb < nk;
            const int ia = wl[ja], ib = vb ? (int)wl[jb] : ia;
            const uint32_t cha = ch[ia], chb = ch[ib], ka = key[ia], kb = key[ib];
            Prop<NW> pa = propose<NW, MODEL>(X_, lab, ch, cz, NM, m + ia, cha, swv(ka), chain);
            Prop<NW> pb = propose<NW, MODEL>(X_, lab, ch, cz, NM, m + ib, chb, swv(kb), chain);
            cnt.prop += 1 + vb;
            cnt.acc += pa.acc + (vb && pb.acc);
            cnt.visits += 1 + vb;
            if (pa.acc) apply<NW, true>(pa, m, lab, ch, cz, par);
            if (vb && pb.acc) apply<NW, true>(pb, m, lab, ch, cz, par);
            key[ia] = 0u;
            if (vb) key[ib] = 0u;
            if (follow) push(rearm(pa, ka), vb ? rearm(pb, kb) : -1);
          }
          // warp-uniform rounds of one proposal per lane (at most one after the paired rounds)
          for (int b0 = j - lane; b0 < nk; b0 += 32) {
            const int jj = b0 + lane;
            int ra = -1;
            if (jj < nk) {
              const int i = wl[jj];
              const uint32_t ki = key[i];
              Prop<NW> p = propose<NW, MODEL>(X_, lab, ch, cz, NM, m + i, ch[i], swv(ki), chain);
              cnt.prop++;
              cnt.visits++;
              if (p.acc) {
                cnt.acc++;
                apply<NW, true>(p, m, lab, ch, cz, par);
              }
              key[i] = 0u;
              ra = rearm(p, ki);
            }
            if (follow) push(ra, -1);
          }
          cnt.busy += nk;
          __syncwarp();
        }
      } else {
        // ---- pre-order: work list of ready nodes (cpu_ref.h:89-126, k_warp :641-700) ----
        // A node's Philox counter {node, sweep, chain} does not depend on the visiting order, so all of
        // the sweep's draws are made up front, 32 nodes at a time, into the key array that par order
        // alone uses: a step of the work list (one latency-bound dependent chain per sweep level of the
        // tree) then reads one word instead of running ten Philox rounds.
        for (int i = lane; i < nint; i += 32) {
          const U4 r = philox10((uint32_t)(m + i), sw, chain, 0u, X_.key0, X_.key1);
          key[i] = (r.y & 0xFFFFFF00u) | (r.x >> 30);
        }
        X_.rtab = key;
        if (lane == 0) wl[0] = (uint16_t)(nint - 1);
        int sp = 1;
        __syncwarp();
        for (int guard = 0; guard <= nint && sp > 0; guard++) {
          int k = min(32, sp), b0 = sp - k;
          int v = lane < k ? m + (int)wl[b0 + lane] : 0;
          __syncwarp();
          uint32_t cw = 0;
          if (lane < k) cw = visit<NW, false, ChainCounters, MODEL, true>(X_, lab, ch, cz, NM, par, v, sw, chain, cnt);
          // internal children become ready (one with two leaf children takes an empty visit next step)
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
        slice_step<NW, ChainCounters, MODEL>(X_, a, lab, ch, cz, cz2, S, sw, chain, lane, cnt);
        NM = not_sliced<NW>(S, X_.slicing);
      }
      __syncwarp();
    }
    cnt.flush(tot);
    // ---- energy of the chain after this launch (fused k_energy) ----
    EvalOut e = eval_w<NW, MODEL>(X_, lab, ch, cz, S, a.leaf_sc, lane);
    if (lane == 0) {
      a.out_lc[c] = e.lcost;
      a.out_sc[c] = e.sc;
      a.out_ns[c] = e.ns;
    }
    __syncwarp();
    if (lane == 0) {
      fence_proxy_async();
      bulk_s2g(a.recs_out + (size_t)c * L.rec_bytes, slot, L.rec_bytes);
      bulk_wait_read();
    }
    __syncwarp();
  }
  if (lane == 0) bulk_wait_all();
  // proposals, accepts and visits are per lane; phases, slice moves and busy lanes are warp-uniform
  unsigned long long v[7] = {tot.prop, tot.acc, tot.steps, tot.visits, tot.sprop, tot.sacc, tot.busy};
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



// ================================================================================================
// k_anneal_pair<NW>: par order with two warps per chain (64 lanes), so that twice as many warps are
// resident for the same shared memory; registers are capped for 14 pairs per SM.  Measured on C2 it is
// 7 % slower than one warp per chain (barrier and atomic overheads outweigh the occupancy), so the plan
// uses it only when asked (kernel_hint 3).  Same chain slot as
// k_anneal_warp plus a second unvisited list: the phase scan compacts with shared-memory atomics
// (entries land in any order; the moves of one phase commute), and the two warps meet at a named
// barrier after the scan and after the visits of every phase.
// ================================================================================================
struct PairSmem {
  uint32_t off_bar, off_cnt, off_leaf, off_slots, slot_bytes, off_scr, total;
  int nint2;
  __host__ __device__ static PairSmem make(const Layout& L, int npairs, int slice_moves) {
    PairSmem w;
    w.nint2 = (int)rnd_up((uint32_t)L.nint, 8);
    w.off_bar = 768;  // [0,256) lse, [256,768) exp
    w.off_cnt = rnd_up(w.off_bar + 8u * (uint32_t)npairs, 16);
    w.off_leaf = rnd_up(w.off_cnt + 32u * (uint32_t)npairs, 128);
    w.off_slots = rnd_up(w.off_leaf + (uint32_t)L.m * (uint32_t)L.nw * 8u, 128);
    // record, then pri / par / wl / U / U2 (u16), then the cz scratch of slice moves
    w.off_scr = L.rec_bytes + 10u * (uint32_t)w.nint2;
    w.slot_bytes = rnd_up(w.off_scr + (slice_moves > 0 ? 4u * (uint32_t)w.nint2 : 0u), 128);
    w.total = w.off_slots + w.slot_bytes * (uint32_t)npairs;
    return w;
  }
};

template <int NW>
__global__ void __launch_bounds__(896, 1) k_anneal_pair(SweepArgs a, int npairs) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = a.L;
  const PairSmem W = PairSmem::make(L, npairs, a.slice_moves);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, pair = warp >> 1, sub = warp & 1;
  const int pl = threadIdx.x & 63;
  const uint32_t bid = 1u + (uint32_t)pair;
  float* s_lse = reinterpret_cast<float*>(smem);
  double* s_exp = reinterpret_cast<double*>(smem + 256);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + W.off_bar);
  int* pc = reinterpret_cast<int*>(smem + W.off_cnt) + 8 * pair;  // [0..2] even phases, [4..6] odd, [7] fail
  uint64_t* s_leaf = reinterpret_cast<uint64_t*>(smem + W.off_leaf);
  for (int t = threadIdx.x; t < 64; t += blockDim.x) {
    s_lse[t] = a.lse_tab[t];
    s_exp[t] = c_exp_tab[t];
  }
  for (int t = threadIdx.x; t < L.m * NW; t += blockDim.x) s_leaf[t] = a.leaf[t];
  if (pl == 0) {
    mbar_init(&s_bar[pair], 1);
    for (int q = 0; q < 8; q++) pc[q] = 0;
  }
  fence_proxy_async();
  __syncthreads();
  auto psync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bid) : "memory"); };

  WarpCtx X_;
  X_.m = L.m;
  X_.nint = L.nint;
  X_.key0 = a.key0;
  X_.key1 = a.key1;
  X_.beta = a.beta;
  X_.sc_target = a.sc_target;
  X_.sc_weight = a.sc_weight;
  X_.slicing = a.slicing;
  X_.exp_device = a.exp_device;
  X_.mode = a.mode;
  X_.mp = a.mp;
  X_.lse = s_lse;
  X_.exptab = s_exp;
  X_.leaf = s_leaf;
  X_.rtab = nullptr;

  uint8_t* slot = smem + W.off_slots + (size_t)pair * W.slot_bytes;
  uint64_t* lab = reinterpret_cast<uint64_t*>(slot);
  uint32_t* ch = reinterpret_cast<uint32_t*>(slot + L.off_ch);
  uint32_t* cz = reinterpret_cast<uint32_t*>(slot + L.off_cz);
  uint64_t* S = reinterpret_cast<uint64_t*>(slot + L.off_S);
  uint16_t* pri = reinterpret_cast<uint16_t*>(slot + L.rec_bytes);
  uint16_t* par = pri + W.nint2;
  uint16_t* wl = par + W.nint2;
  uint16_t* Ua = wl + W.nint2;
  uint16_t* Ub = Ua + W.nint2;
  uint32_t* cz2 = reinterpret_cast<uint32_t*>(slot + W.off_scr);
  const int m = L.m, nint = L.nint, nint2 = W.nint2;
  const unsigned FULL = 0xFFFFFFFFu;
  const unsigned lt = (1u << lane) - 1u;
  Counters cnt{};
  uint32_t phase = 0;

  for (int c = blockIdx.x * npairs + pair; c < a.nchains; c += gridDim.x * npairs) {
    uint8_t* grec = a.recs + (size_t)c * L.rec_bytes;
    if (pl == 0) {
      fence_proxy_async();
      mbar_expect_tx(&s_bar[pair], L.rec_bytes);
      if (!a.debug_arm_only) bulk_g2s(slot, grec, L.rec_bytes, &s_bar[pair]);
    }
    bool ok = mbar_wait(&s_bar[pair], phase, a.wait_cycles);
    phase ^= 1u;
    const bool all_ok = __all_sync(FULL, ok);
    if (lane == 0 && !all_ok) atomicOr(&pc[7], 1);
    psync();
    if (pc[7]) {
      if (pl == 0) atomicExch(a.err, 1);
      break;
    }
    const uint32_t chain = (uint32_t)(a.chain0 + c);
    const uint32_t hc = chain_hash(chain, a.key0);
    for (int i = pl; i < nint; i += 64) {
      uint32_t cw = ch[i];
      int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
      if (l >= m) par[l - m] = (uint16_t)(m + i);
      if (r >= m) par[r - m] = (uint16_t)(m + i);
    }
    if (pl == 0) par[nint - 1] = 0xFFFFu;
    psync();
    for (int s = 0; s < a.nsweeps; s++) {
      const uint32_t sw = a.sweep0 + (uint32_t)s;
      const uint32_t hs = sweep_hash(sw, hc);
      for (int i = pl; i < nint; i += 64) {
        pri[i] = (uint16_t)node_pri((uint32_t)(m + i), hs);
        Ua[i] = (uint16_t)i;
      }
      uint16_t *U = Ua, *U2 = Ub;
      int nU = nint;
      psync();
      const Set<NW> NM = not_sliced<NW>(S, X_.slicing);
      for (int ph = 0; ph <= nint; ph++) {
        int* cur = pc + 4 * (ph & 1);
        int* nxt = pc + 4 * ((ph + 1) & 1);
        for (int base = 0; base < nU; base += 64) {
          int j = base + pl;
          bool valid = j < nU;
          int i = valid ? (int)U[j] : 0;
          bool act = false;
          uint32_t cw = 0;
          if (valid) {
            uint32_t key = ((uint32_t)pri[i] << 16) | (uint32_t)(m + i);
            act = true;
            int p = par[i];
            if (p != 0xFFFF) {
              uint32_t pp = pri[p - m];
              if (pp && ((pp << 16) | (uint32_t)p) > key) act = false;
            }
            cw = ch[i];
            int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
            if (act && l >= m) {
              uint32_t pq = pri[l - m];
              if (pq && ((pq << 16) | (uint32_t)l) > key) act = false;
            }
            if (act && r >= m) {
              uint32_t pq = pri[r - m];
              if (pq && ((pq << 16) | (uint32_t)r) > key) act = false;
            }
          }
          bool cher = act && (int)(cw & 0xFFFFu) < m && (int)(cw >> 16) < m;
          bool prop = act && !cher;
          bool keep = valid && !act;
          unsigned ba = __ballot_sync(FULL, prop), bc = __ballot_sync(FULL, cher), bk = __ballot_sync(FULL, keep);
          int p0 = 0, p1 = 0, p2 = 0;
          if (lane == 0) {
            if (ba) p0 = atomicAdd(&cur[0], __popc(ba));
            if (bc) p1 = atomicAdd(&cur[1], __popc(bc));
            if (bk) p2 = atomicAdd(&cur[2], __popc(bk));
          }
          p0 = __shfl_sync(FULL, p0, 0);
          p1 = __shfl_sync(FULL, p1, 0);
          p2 = __shfl_sync(FULL, p2, 0);
          if (prop) wl[p0 + __popc(ba & lt)] = (uint16_t)i;
          if (cher) wl[nint2 - 1 - (p1 + __popc(bc & lt))] = (uint16_t)i;
          if (keep) U2[p2 + __popc(bk & lt)] = (uint16_t)i;
        }
        if (pl == 0) {
          nxt[0] = 0;
          nxt[1] = 0;
          nxt[2] = 0;
        }
        psync();
        const int nk = cur[0], nc = cur[1];
        nU = cur[2];
        uint16_t* tmp = U;
        U = U2;
        U2 = tmp;
        if (nk + nc == 0) break;
        if (pl == 0) {
          cnt.steps++;
          cnt.busy += nk;
        }
        for (int j = pl; j < nc; j += 64) {
          pri[wl[nint2 - 1 - j]] = 0;
          cnt.visits++;
        }
        for (int j = pl; j < nk; j += 64) {
          int i = wl[j];
          visit<NW, true>(X_, lab, ch, cz, NM, par, m + i, sw, chain, cnt);
          pri[i] = 0;
          cnt.visits++;
        }
        psync();
      }
      if (a.slice_moves > 0 && (sw + 1) % (uint32_t)a.slice_every == 0) {
        if (sub == 0) slice_step<NW>(X_, a, lab, ch, cz, cz2, S, sw, chain, lane, cnt);
        psync();
      }
    }
    if (sub == 0) {
      EvalOut e = eval_cached<NW>(X_, cz, S, a.leaf_sc, lane);
      if (lane == 0) {
        a.out_lc[c] = e.lcost;
        a.out_sc[c] = e.sc;
        a.out_ns[c] = e.ns;
      }
    }
    psync();
    if (pl == 0) {
      fence_proxy_async();
      bulk_s2g(a.recs_out + (size_t)c * L.rec_bytes, slot, L.rec_bytes);
      bulk_wait_read();
    }
    psync();
  }
  if (pl == 0) bulk_wait_all();
  // proposals, accepts, visits per lane; phases, busy lanes once per pair; slice moves by all of warp 0
  unsigned long long v[7] = {cnt.prop, cnt.acc, cnt.steps, cnt.visits, cnt.sprop, cnt.sacc, cnt.busy};
  for (int o = 16; o > 0; o >>= 1) {
    v[0] += __shfl_xor_sync(FULL, v[0], o);
    v[1] += __shfl_xor_sync(FULL, v[1], o);
    v[3] += __shfl_xor_sync(FULL, v[3], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < 7; q++)
      if (v[q]) atomicAdd(&a.stats[q], v[q]);
  }
}

// ================================================================================================
// k_anneal_block: one CTA per chain for chains that do not fit in shared memory.  Per-node metadata
// (children, (cost, size), chunk summaries, priorities, parents, work lists) in shared memory; label
// sets stay in HBM and are streamed in 16-byte chunks by G lanes per node (the reference's visit_coop,
// csrc/treesa_gpu.cu:267-373, with u64 words and an exact integer cost cache).
// ================================================================================================
// With chunk summaries, a par phase is processed as a flat list of (node, chunk) items spread evenly over
// the CTA's threads (see par_phase_flat); these are its per-batch tables.
constexpr int kFlatBatch = 512;            // nodes per batch (one owner thread each)
constexpr int kFlatItems = 8192;           // (node, chunk) items per window
// a batch of at most kFlatDirect items per thread decodes each item's node by a binary search over the
// owners' item offsets; larger batches build the item list first (flat_build).  Measured on C3/C4: 2
// against 1 and 0 (always the list), 1 % and 2-4 % faster.
constexpr int kFlatDirect = 2;
constexpr uint32_t kLeafSumCache = 220u << 10;  // cache leaf summaries in shared memory below this total

struct BlockSmem {
  uint32_t off_ch, off_cz, off_cz2, off_sum, off_S, off_pri, off_par, off_wl, off_U, off_U2, total;
  uint32_t off_ninfo, off_nrnd, off_ncnt, off_nxs, off_nacc, off_noff, off_nu, off_scan, off_lsum, off_items;
  int nint2;
  // pair: the layout of k_anneal_cluster, which also keeps the leaf chunk summaries in shared memory (its
  // label loads bypass L1; the single-CTA kernel leaves that room to L1, which serves its reloads)
  // gmeta 1: the children, cost and summary words are read and written in the chain record in global
  // memory (networks whose per-node metadata does not fit in shared memory); gmeta 2: also no unvisited
  // lists, no flat-phase tables and no slice-move scratch in shared memory (the largest networks)
  __host__ __device__ static BlockSmem make(const Layout& L, int slice_moves, bool pair = false,
                                            int gmeta = 0) {
    BlockSmem b;
    b.nint2 = (int)rnd_up((uint32_t)L.nint, 8);
    const uint32_t n2 = (uint32_t)b.nint2;
    uint32_t o = 1024;  // [0,256) lse, [256,768) exp, [768,1024) block scalars
    b.off_ch = b.off_cz = b.off_sum = 0;
    if (!gmeta) {
      b.off_ch = o;
      o += 4 * n2;
      b.off_cz = o;
      o += 4 * n2;
    }
    b.off_cz2 = o;
    if (slice_moves > 0 && gmeta < 2) o += 4 * n2;
    if (!gmeta) {
      b.off_sum = o;
      if (L.sums) o += 8 * n2;
    }
    b.off_S = rnd_up(o, 16);
    o = b.off_S + rnd_up(8u * (uint32_t)L.nw, 16);
    // pri and wl are adjacent, and so are U and U2: read as two arrays of n2 words they hold the depth
    // computation of par_band at the start of a sweep
    b.off_par = o;
    o += 2 * n2;
    b.off_pri = o;
    o += 2 * n2;
    b.off_wl = o;
    o += 2 * n2;
    b.off_U = b.off_U2 = 0;
    if (gmeta < 2) {
      b.off_U = o;
      o += 2 * n2;
      b.off_U2 = o;
      o += 2 * n2;
    }
    if (L.sums && gmeta < 2) {
      o = rnd_up(o, 16);
      b.off_ninfo = o;
      o += 8 * kFlatBatch;
      b.off_ncnt = o;
      o += 8 * kFlatBatch;
      b.off_nxs = o;
      o += 8 * kFlatBatch;
      b.off_nu = o;
      o += 8 * kFlatBatch;
      b.off_nrnd = o;
      o += 4 * kFlatBatch;
      b.off_noff = o;
      o += 4 * kFlatBatch;
      b.off_items = o;
      o += 4 * kFlatItems;
      b.off_scan = o;
      o += 4 * 32;
      b.off_nacc = o;
      o += kFlatBatch;
      // leaf chunk summaries, when they fit (otherwise read from global memory)
      o = rnd_up(o, 16);
      b.off_lsum = 0;
      if (pair && o + 8u * (uint32_t)L.m <= kLeafSumCache) {
        b.off_lsum = o;
        o += 8u * (uint32_t)L.m;
      }
    } else {
      b.off_ninfo = b.off_ncnt = b.off_nxs = b.off_nrnd = b.off_noff = b.off_nu = b.off_scan = b.off_nacc = 0;
      b.off_lsum = b.off_items = 0;
    }
    b.total = rnd_up(o, 128);
    return b;
  }
};

struct BlkCtx {
  int m, nint, nw, nchunks;
  uint32_t key0, key1;
  float beta, sc_target, sc_weight;
  int slicing, exp_device;
  int mode;  // energy mode of the launch (the model kernels: 1 gpu, 2 h100)
  ModelParams mp;
  const float* lse;          // shared
  const double* exptab;      // shared
  const uint64_t* leaf;      // global [m][nw]
  const uint64_t* leaf_sum;  // global [m]
  uint64_t* lab;             // global: this chain's label sets
  uint32_t* ch;              // shared
  uint32_t* cz;              // shared
  uint64_t* sum;             // shared (when sums)
  uint64_t* S;               // shared copy of the slice set
};

__device__ __forceinline__ ulonglong2 ld2(const uint64_t* p) { return *reinterpret_cast<const ulonglong2*>(p); }
// 16-byte global load cached in L2 only: label sets that the other CTA of a cluster rewrites are never
// read from a stale L1 line
__device__ __forceinline__ ulonglong2 ld2_cg(const uint64_t* p) {
  ulonglong2 r;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];"
               : "=l"(r.x), "=l"(r.y)
               : "l"((unsigned long long)__cvta_generic_to_global(p))
               : "memory");
  return r;
}
// Split cluster barrier: arrive (release) after the phase's scan, wait (acquire) before the first write
// into the other CTA's shared memory.  Every thread of both CTAs executes each, in the same order.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// The other CTA's copies of the replicated per-node arrays of a CTA pair, each mapped with
// map_shared_rank (distributed shared memory; null for a single CTA).  Always indexed from these bases:
// a local shared-memory pointer plus an offset would keep the shared state space and miss the peer.
struct PeerArrays {
  uint32_t* ch;
  uint32_t* cz;
  uint64_t* sum;
  uint16_t* par;
  uint16_t* pri;
};
// element i of a replicated array in this CTA and, for a CTA pair, in the other CTA
template <typename T>
__device__ __forceinline__ void mset(T* local, T* peer, int i, T v) {
  local[i] = v;
  if (peer) peer[i] = v;
}

// lanes t, t+G, ... of the set chunks of u (SUMS) or of all chunks
template <bool SUMS, typename F>
__device__ __forceinline__ void for_chunks(uint64_t u, int nchunks, int G, int t, F&& f) {
  if (SUMS) {
    int k = 0;
    while (u) {
      int c = __ffsll((long long)u) - 1;
      u &= u - 1;
      if ((k & (G - 1)) == t) f(c);
      k++;
    }
  } else {
#pragma unroll 4
    for (int c = t; c < nchunks; c += G) f(c);
  }
}

// par_follow state of a CTA's sweep: an accepted first visit re-arms its pivot child P (if the sweep
// already visited it) with an even priority and appends P to the unvisited list U at *nU
// (cpu_ref.h:168-175).
struct FollowCtx {
  uint16_t* pri;
  uint16_t* U;
  int* nU;
  uint32_t hs;
};
__device__ __forceinline__ void follow_rearm(const FollowCtx* f, int Pn, int m) {
  if (f && f->pri[Pn - m] == 0) {
    f->pri[Pn - m] = (uint16_t)follow_pri((uint32_t)Pn, f->hs);
    if (f->U) f->U[atomicAdd(f->nU, 1)] = (uint16_t)(Pn - m);  // no list: the full scan finds it
  }
}

// sweep: the Philox sweep counter of this visit; fol: re-arm on accept (a first visit with par_follow)
template <bool SUMS, bool PAR, bool MODEL = false>
__device__ __forceinline__ void visit_coop(const BlkCtx& B, uint16_t* par, int v, uint32_t sweep, uint32_t chain,
                                           int G, int t, unsigned gm, BlkCounters& cnt,
                                           const FollowCtx* fol = nullptr) {
  const int m = B.m, i = v - m, nw = B.nw;
  uint32_t chv = B.ch[i];
  int l = (int)(chv & 0xFFFFu), r = (int)(chv >> 16);
  bool li = l >= m, ri = r >= m;
  if (!li && !ri) return;
  U4 rnd = philox10((uint32_t)v, sweep, chain, 0u, B.key0, B.key1);
  int rule = pick_rule(li, ri, rnd.x);
  int slotP = rule >> 1;
  int slotM = ((rule ^ (rule >> 1)) & 1) ^ 1;
  int Pn = slotP ? r : l, On = slotP ? l : r;
  uint32_t chp = B.ch[Pn - m];
  int Mn = slotM ? (int)(chp >> 16) : (int)(chp & 0xFFFFu);
  int Kn = slotM ? (int)(chp & 0xFFFFu) : (int)(chp >> 16);
  const uint64_t* gD = B.lab + (size_t)i * nw;
  uint64_t* gP = B.lab + (size_t)(Pn - m) * nw;
  const uint64_t* gO = On >= m ? B.lab + (size_t)(On - m) * nw : B.leaf + (size_t)On * nw;
  const uint64_t* gK = Kn >= m ? B.lab + (size_t)(Kn - m) * nw : B.leaf + (size_t)Kn * nw;
  const uint64_t* gM = Mn >= m ? B.lab + (size_t)(Mn - m) * nw : B.leaf + (size_t)Mn * nw;
  uint64_t u = ~0ull;
  if (SUMS) {
    auto so = [&](int n) { return n >= m ? B.sum[n - m] : B.leaf_sum[n]; };
    u = B.sum[i] | so(On) | so(Kn) | so(Mn);
  }
  int sx = 0, k2 = 0, k3 = 0;
  C4 cc[4] = {};  // MODEL: (K,M)->P, (P,O)->D, (K,O)->X, (X,M)->D
  for_chunks<SUMS>(u, B.nchunks, G, t, [&](int c) {
    ulonglong2 d = ld2(gD + 2 * c), o = ld2(gO + 2 * c), k = ld2(gK + 2 * c), mm = ld2(gM + 2 * c);
    uint64_t n0 = ~0ull, n1 = ~0ull;
    if (B.slicing) {
      n0 = ~B.S[2 * c];
      n1 = ~B.S[2 * c + 1];
    }
    uint64_t x0 = (k.x | o.x) & (mm.x | d.x), x1 = (k.y | o.y) & (mm.y | d.y);
    uint64_t xm0 = x0 & n0, xm1 = x1 & n1;
    sx += __popcll(xm0) + __popcll(xm1);
    k2 += __popcll(k.x & o.x & ~x0 & n0) + __popcll(k.y & o.y & ~x1 & n1);
    k3 += __popcll(xm0 & mm.x & ~d.x) + __popcll(xm1 & mm.y & ~d.y);
    if constexpr (MODEL) {
      const ulonglong2 pp = ld2(gP + 2 * c);
      count3(k.x & n0, mm.x & n0, pp.x & n0, cc[0]);
      count3(k.y & n1, mm.y & n1, pp.y & n1, cc[0]);
      count3(pp.x & n0, o.x & n0, d.x & n0, cc[1]);
      count3(pp.y & n1, o.y & n1, d.y & n1, cc[1]);
      count3(k.x & n0, o.x & n0, xm0, cc[2]);
      count3(k.y & n1, o.y & n1, xm1, cc[2]);
      count3(xm0, mm.x & n0, d.x & n0, cc[3]);
      count3(xm1, mm.y & n1, d.y & n1, cc[3]);
    }
  });
  for (int off = G >> 1; off > 0; off >>= 1) {
    sx += __shfl_xor_sync(gm, sx, off);
    k2 += __shfl_xor_sync(gm, k2, off);
    k3 += __shfl_xor_sync(gm, k3, off);
    if constexpr (MODEL) {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        cc[q].B += __shfl_xor_sync(gm, cc[q].B, off);
        cc[q].M += __shfl_xor_sync(gm, cc[q].M, off);
        cc[q].N += __shfl_xor_sync(gm, cc[q].N, off);
        cc[q].K += __shfl_xor_sync(gm, cc[q].K, off);
      }
    }
  }
  uint32_t czv = B.cz[i], czp = B.cz[Pn - m];
  int sd = (int)(czv & 0xFFFFu), sp = (int)(czp & 0xFFFFu);
  int cP1 = sx + k2, cV1 = sd + k3;
  float dE;
  if constexpr (MODEL) {
    auto cost = [&](const C4& q) { return model_cost(B.mode, B.mp, q.B, q.M, q.N, q.K); };
    dE = model_energy(lse_f(cost(cc[0]), cost(cc[1])), lse_f(cost(cc[2]), cost(cc[3])), sp, sd, sx, B.sc_target,
                      B.sc_weight);
  } else {
    dE = move_energy((int)(czp >> 16), (int)(czv >> 16), sp, sd, sx, cP1, cV1, B.sc_target, B.sc_weight, B.lse);
  }
  bool acc = accept_rt(B.exp_device, B.beta, B.exptab, rnd.y, dE);
  const int nck = SUMS ? __popcll(u) : B.nchunks;
  if (t == 0) {
    cnt.prop++;
    cnt.chunks += nck;
    if (acc) cnt.chunks_acc += nck;
  }
  if (!acc) return;
  uint64_t xs = 0;
  for_chunks<SUMS>(u, B.nchunks, G, t, [&](int c) {
    ulonglong2 d = ld2(gD + 2 * c), o = ld2(gO + 2 * c), k = ld2(gK + 2 * c), mm = ld2(gM + 2 * c);
    ulonglong2 x = make_ulonglong2((k.x | o.x) & (mm.x | d.x), (k.y | o.y) & (mm.y | d.y));
    *reinterpret_cast<ulonglong2*>(gP + 2 * c) = x;
    if (x.x | x.y) xs |= 1ull << c;
  });
  if (SUMS)
    for (int off = G >> 1; off > 0; off >>= 1) xs |= __shfl_xor_sync(gm, xs, off);
  __syncwarp(gm);
  if (t == 0) {
    cnt.acc++;
    uint32_t nchp = slotM ? ((chp & 0xFFFFu) | ((uint32_t)On << 16)) : ((chp & 0xFFFF0000u) | (uint32_t)On);
    uint32_t nchv = slotP ? ((chv & 0xFFFF0000u) | (uint32_t)Mn) : ((chv & 0xFFFFu) | ((uint32_t)Mn << 16));
    B.ch[Pn - m] = nchp;
    B.ch[i] = nchv;
    B.cz[Pn - m] = ((uint32_t)cP1 << 16) | (uint32_t)sx;
    B.cz[i] = ((uint32_t)cV1 << 16) | (uint32_t)sd;
    if (SUMS) B.sum[Pn - m] = xs;
    if (PAR) {
      if (On >= m) par[On - m] = (uint16_t)Pn;
      if (Mn >= m) par[Mn - m] = (uint16_t)v;
    }
    follow_rearm(fol, Pn, m);
  }
}

// Model modes: log2 cost of every internal node's contraction, counted from the label sets in HBM on the
// network sliced by B.S, by all threads of the CTA into costs[] (then read by eval_cz).
__device__ void block_model_costs(const BlkCtx& B, float* costs) {
  const int m = B.m, nw = B.nw;
  for (int i = threadIdx.x; i < B.nint; i += blockDim.x) {
    const uint32_t cw = B.ch[i];
    const int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
    const uint64_t* x = l >= m ? B.lab + (size_t)(l - m) * nw : B.leaf + (size_t)l * nw;
    const uint64_t* y = r >= m ? B.lab + (size_t)(r - m) * nw : B.leaf + (size_t)r * nw;
    const uint64_t* z = B.lab + (size_t)i * nw;
    C4 c{};
    for (int w = 0; w < nw; w++) {
      const uint64_t nm = B.slicing ? ~B.S[w] : ~0ull;
      count3(x[w] & nm, y[w] & nm, z[w] & nm, c);
    }
    costs[i] = model_cost(B.mode, B.mp, c.B, c.M, c.N, c.K);
  }
  __syncthreads();
}

// Whole-chain energy from a (cost, size) cache, one warp, in the reference's lane order.
// costs: the nodes' log2 costs in the model modes (block_model_costs), null for tc (from cz)
__device__ EvalOut eval_cz(const uint32_t* cz, int nint, const uint64_t* S, int nw, const uint64_t* leaf, int m,
                           int slicing, int leaf_sc, int lane, const float* costs = nullptr) {
  const unsigned FULL = 0xFFFFFFFFu;
  float acc = -INFINITY;
  int scl = 0, cntl = 0;
  for (int i = lane; i < nint; i += 32) {
    uint32_t w = cz[i];
    int Z = (int)(w & 0xFFFFu);
    acc = lse_f(acc, costs ? costs[i] : (float)(int)(w >> 16));
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
  if (slicing)
    for (int w = lane; w < nw; w += 32) ns += __popcll(S[w]);
  for (int o = 16; o > 0; o >>= 1) {
    cnt += __shfl_xor_sync(FULL, cnt, o);
    ns += __shfl_xor_sync(FULL, ns, o);
  }
  int sc = max(scmax, leaf_sc);
  if (slicing && leaf_sc > scmax) {
    int ll = 0;
    for (int i = lane; i < m; i += 32) {
      int Z = 0;
      for (int w = 0; w < nw; w++) Z += __popcll(leaf[(size_t)i * nw + w] & ~S[w]);
      ll = max(ll, Z);
    }
    for (int o = 16; o > 0; o >>= 1) ll = max(ll, __shfl_xor_sync(FULL, ll, o));
    sc = max(scmax, ll);
  }
  return EvalOut{acc, sc, scmax, cnt, ns};
}

__device__ __forceinline__ int nth_label_rt(const uint64_t* A, const uint64_t* S, int nw, int n) {
  for (int w = 0; w < nw; w++) {
    uint64_t x = A[w] & (S ? ~S[w] : ~0ull);
    int c = __popcll(x);
    if (n < c) {
      for (int k = 0; k < n; k++) x &= x - 1;
      return w * 64 + __ffsll((long long)x) - 1;
    }
    n -= c;
  }
  return -1;
}

// Slice moves of one chain, the whole CTA cooperating (slice_step, csrc/treesa_gpu.cu:445-502):
// warp 0 chooses and judges the proposals; all threads recompute the (cost, size) cache for the
// proposed slice set.
// costs: scratch for the model modes' node costs (null in tc mode)
__device__ void slice_step_block(const BlkCtx& B, const SweepArgs& a, uint32_t* cz2, int* sh, float* shf,
                                 uint32_t sweep, uint32_t chain, BlkCounters& cnt, float* costs = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, T = blockDim.x, m = B.m, nw = B.nw;
  EvalOut cur{};
  float Ecur = 0.f;
  if (costs) block_model_costs(B, costs);
  if (warp == 0) {
    cur = eval_cz(B.cz, B.nint, B.S, nw, B.leaf, m, B.slicing, a.leaf_sc, lane, costs);
    Ecur = slice_energy(cur, B.sc_target, B.sc_weight);
  }
  for (int j = 0; j < a.slice_moves; j++) {
    if (warp == 0) {
      U4 r1 = philox10(0x10000u + 2u * j, sweep, chain, 0u, B.key0, B.key1);
      int type;
      if (cur.ns == 0) type = 0;
      else if (cur.ns >= a.max_slices) type = (r1.x >> 31) ? 1 : 2;
      else type = r1.x < 0x80000000u ? 0 : (r1.x < 0xC0000000u ? 1 : 2);
      int ladd = -1, lrem = -1;
      if (type != 1 && cur.ncand > 0 && cur.sc_int > 0) {
        int rr = (int)(r1.y % (uint32_t)cur.ncand), node = -1;
        for (int base = 0; base < B.nint && node < 0; base += 32) {
          int i = base + lane;
          int Z = i < B.nint ? (int)(B.cz[i] & 0xFFFFu) : -1;
          unsigned bb = __ballot_sync(0xFFFFFFFFu, Z == cur.sc_int);
          int c = __popc(bb);
          if (rr < c) {
            for (int k = 0; k < rr; k++) bb &= bb - 1;
            node = base + __ffs(bb) - 1;
          } else {
            rr -= c;
          }
        }
        if (node >= 0) ladd = nth_label_rt(B.lab + (size_t)node * nw, B.S, nw, (int)(r1.z % (uint32_t)cur.sc_int));
      }
      if (type != 0) lrem = nth_label_rt(B.S, nullptr, nw, (int)(r1.w % (uint32_t)cur.ns));
      if (type == 2 && ladd < 0) type = 1;
      int skip = (type == 0 && ladd < 0);
      if (lane == 0) {
        sh[0] = skip;
        sh[1] = type;
        sh[2] = ladd;
        sh[3] = lrem;
        if (!skip) {
          if (type != 1) B.S[ladd >> 6] |= 1ull << (ladd & 63);
          if (type != 0) B.S[lrem >> 6] &= ~(1ull << (lrem & 63));
        }
      }
    }
    __syncthreads();
    if (sh[0]) {
      __syncthreads();
      continue;
    }
    for (int i = tid; i < B.nint; i += T) {
      uint32_t cw = B.ch[i];
      int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
      const uint64_t* px = l >= m ? B.lab + (size_t)(l - m) * nw : B.leaf + (size_t)l * nw;
      const uint64_t* py = r >= m ? B.lab + (size_t)(r - m) * nw : B.leaf + (size_t)r * nw;
      const uint64_t* pz = B.lab + (size_t)i * nw;
      int Z = 0, K = 0;
      for (int w = 0; w < nw; w++) {
        uint64_t nm = ~B.S[w], zz = pz[w] & nm;
        Z += __popcll(zz);
        K += __popcll(px[w] & py[w] & nm & ~zz);
      }
      cz2[i] = ((uint32_t)(Z + K) << 16) | (uint32_t)Z;
    }
    __syncthreads();
    if (costs) block_model_costs(B, costs);  // on the proposed slice set
    if (warp == 0) {
      EvalOut nxt = eval_cz(cz2, B.nint, B.S, nw, B.leaf, m, B.slicing, a.leaf_sc, lane, costs);
      float Enew = slice_energy(nxt, B.sc_target, B.sc_weight);
      U4 r2 = philox10(0x10001u + 2u * j, sweep, chain, 0u, B.key0, B.key1);
      bool acc = accept_rt(B.exp_device, B.beta, B.exptab, r2.x, __fsub_rn(Enew, Ecur));
      cnt.sprop++;
      if (acc) {
        cnt.sacc++;
        cur = nxt;
        Ecur = Enew;
      }
      if (lane == 0) sh[4] = acc;
    }
    __syncthreads();
    if (sh[4]) {
      for (int i = tid; i < B.nint; i += T) B.cz[i] = cz2[i];
    } else if (tid == 0) {
      int type = sh[1], ladd = sh[2], lrem = sh[3];
      if (type != 1) B.S[ladd >> 6] &= ~(1ull << (ladd & 63));
      if (type != 0) B.S[lrem >> 6] |= 1ull << (lrem & 63);
    }
    __syncthreads();
  }
  (void)shf;
}

// One par phase's scan of a CTA's unvisited list U[0, nU) (csrc/cpu_ref.h:154-166): a node is active iff
// its key pri << 16 | id exceeds the key of every unvisited neighbour (parent, internal children; a
// visited node has pri 0, so its key is below every unvisited key).  Active nodes are appended to wl,
// the others to U2, at places reserved through the counters ctr[0] and ctr[1].  Each thread takes up to R
// entries per round with all their shared-memory loads issued together (a missing neighbour reads the
// node's own key, which blocks nothing), and a warp reserves its places for the whole round with one
// atomic per list.
// LIST = false: no lists; every node [0, nU) is an entry, the visited ones (pri 0) skipped, and no kept
// list is written (U and U2 unused).
template <int R, bool LIST = true>
__device__ __forceinline__ void phase_scan(const uint16_t* U, int nU, uint16_t* wl, uint16_t* U2, int* ctr,
                                           const uint16_t* pri, const uint16_t* par, const uint32_t* ch, int m) {
  const int tid = threadIdx.x, T = blockDim.x, lane = tid & 31;
  const unsigned FULL = 0xFFFFFFFFu, lt = (1u << lane) - 1u;
  for (int base = 0; base < nU; base += R * T) {
    int q[R];
    bool valid[R], act[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int j = base + r * T + tid;
      if (LIST) {
        valid[r] = j < nU;
        q[r] = valid[r] ? (int)U[j] : 0;
      } else {
        q[r] = j < nU ? j : 0;
        valid[r] = j < nU && pri[q[r]] != 0;
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t own = (uint32_t)(m + q[r]);
      const uint32_t key = ((uint32_t)pri[q[r]] << 16) | own;
      const int p = par[q[r]];
      const uint32_t cw = ch[q[r]];
      const int l = (int)(cw & 0xFFFFu), rr = (int)(cw >> 16);
      const uint32_t np = p != 0xFFFF ? (uint32_t)p : own, nl = l >= m ? (uint32_t)l : own,
                     nr = rr >= m ? (uint32_t)rr : own;
      const uint32_t kp = ((uint32_t)pri[np - m] << 16) | np, kl = ((uint32_t)pri[nl - m] << 16) | nl,
                     kr = ((uint32_t)pri[nr - m] << 16) | nr;
      act[r] = valid[r] && key >= kp && key >= kl && key >= kr;  // ids differ: equal only for the node itself
    }
    unsigned ba[R], bk[R];
    int ta = 0, tk = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
      ba[r] = __ballot_sync(FULL, act[r]);
      bk[r] = __ballot_sync(FULL, valid[r] && !act[r]);
      ta += __popc(ba[r]);
      tk += __popc(bk[r]);
    }
    int pa = 0, pk = 0;
    if (lane == 0) {
      if (ta) pa = atomicAdd(&ctr[0], ta);
      if (LIST && tk) pk = atomicAdd(&ctr[1], tk);
    }
    pa = __shfl_sync(FULL, pa, 0);
    pk = __shfl_sync(FULL, pk, 0);
#pragma unroll
    for (int r = 0; r < R; r++) {
      if (act[r]) wl[pa + __popc(ba[r] & lt)] = (uint16_t)q[r];
      if (LIST && valid[r] && !act[r]) U2[pk + __popc(bk[r] & lt)] = (uint16_t)q[r];
      pa += __popc(ba[r]);
      pk += __popc(bk[r]);
    }
  }
}

__device__ __forceinline__ int pick_group(int k, int T) {
  int G = 32;
  while (G > 1 && k * G > T) G >>= 1;
  return G;
}

// ------------------------------------------------------------------------------------------------
// One par phase of a chain with chunk summaries, as a flat list of (node, chunk) items.
//
// The label sets of a move touch a data-dependent number of 16-byte chunks (from one to the whole set),
// so handing each node to a fixed group of lanes leaves the phase waiting for its widest node, one
// dependent HBM/L2 round trip per chunk.  Here the phase's nodes are taken in batches of kFlatBatch:
//   1. one owner thread per node draws the rule (Philox), finds P, O, K, M and the chunk union u;
//   2. a block-wide exclusive scan of popc(u) numbers the batch's chunk items;
//   3. every thread takes items e = tid, tid + T, ... (IPT at a time, all 4 IPT 16-byte loads issued
//      before any is used), finds each item's node by a binary search over the batch's item offsets
//      and its chunk as the k-th set bit of u, and adds the item's popcounts (sx | k2 << 16, k3) and
//      nonzero bit of X into the node's shared-memory totals with 32-bit atomics;
//   4. the owner evaluates dE and the Metropolis test and rewrites the node's metadata on accept;
//   5. X is stored into P's chunks for the items of accepted nodes (a thread's first IPT items from
//      registers, any further ones recomputed: the sets they read are unchanged by the phase).
// Same moves, same random numbers and the same integer counts as visit_coop, so the chains are
// bit-identical; only the schedule of the loads changes.
// ------------------------------------------------------------------------------------------------
struct FlatTabs {
  uint2* info;    // [batch] Pn | On << 16, Kn | Mn << 16 (x = ~0: leaf-only node)
  uint32_t* rnd;  // [batch] Philox .y of the proposal
  uint2* cnt;     // [batch] counts: x = sx | k2 << 16, y = k3 (each at most 64 * 128)
  uint2* xs;      // [batch] chunk summary of X: x = chunks 0-31, y = chunks 32-63
  uint8_t* acc;   // [batch] accepted
  uint32_t* off;  // [batch] number of the node's first item
  uint64_t* u;    // [batch] chunk union of the node's four sets
  uint32_t* items;  // [window] node << 16 | chunk
  int* scan;      // [32] per-warp totals
};

struct Item {
  int j, c;  // node of the batch, chunk
};
__device__ __forceinline__ Item item_of(uint32_t it) { return Item{(int)(it >> 16), (int)(it & 0xFFFFu)}; }

// position of the k-th (0-based) set bit of x; k < popc(x)
__device__ __forceinline__ int nth_bit32(uint32_t x, int k) {
  int pos = 0;
#pragma unroll
  for (int w = 16; w > 0; w >>= 1) {
    const int c = __popc(x & ((1u << w) - 1u));
    if (k >= c) {
      k -= c;
      x >>= w;
      pos += w;
    }
  }
  return pos;
}
// Item e of a batch of nb nodes found without a list: the last node whose first item is <= e (nodes without
// items share their successor's offset and are never returned for a valid e), its chunk the k-th set bit
// of its union.  Used when a batch has at most two items per thread, where it saves the list's build and
// barrier; wider batches read the list (flat_build).
__device__ __forceinline__ Item flat_decode(const FlatTabs& F, int nb, int e) {
  int lo = 0, hi = nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int)F.off[mid] <= e) lo = mid;
    else hi = mid - 1;
  }
  const int k = e - (int)F.off[lo];
  const uint64_t u = F.u[lo];
  const uint32_t ul = (uint32_t)u;
  const int nl = __popc(ul);
  return Item{lo, k < nl ? nth_bit32(ul, k) : 32 + nth_bit32((uint32_t)(u >> 32), k - nl)};
}

// The items numbered [w0, w0 + kFlatItems) into F.items.  A warp whose owners have fewer than 32 chunks
// each lets every owner write its own items (as many steps as the widest owner has chunks); otherwise
// the warp expands the masks of its 32 owners together: for owner o (mask and offset broadcast from its
// lane), lane l writes the item of chunk l (and 32 + l) if that bit is set, at the owner's offset plus
// the number of set bits below it.
__device__ __forceinline__ void flat_build(const FlatTabs& F, int nb, int w0) {
  const int tid = threadIdx.x, lane = tid & 31, wbase = tid & ~31;
  const uint32_t lt = (1u << lane) - 1u;
  const unsigned FULL = 0xFFFFFFFFu;
  const uint64_t myu = tid < nb ? F.u[tid] : 0ull;
  const int myoff = (int)(tid < nb ? F.off[tid] : 0u) - w0;
  int wide = __popcll(myu);
  for (int o = 16; o > 0; o >>= 1) wide = max(wide, __shfl_xor_sync(FULL, wide, o));
  if (wide < 32) {
    uint64_t uu = myu;
    for (int k = myoff; uu; k++) {
      const int c = __ffsll((long long)uu) - 1;
      uu &= uu - 1;
      if (k >= 0 && k < kFlatItems) F.items[k] = ((uint32_t)tid << 16) | (uint32_t)c;
    }
    return;
  }
  const int nown = min(32, nb - wbase);  // warp-uniform
  for (int o = 0; o < nown; o++) {
    const int j = wbase + o;
    const uint64_t u = __shfl_sync(FULL, myu, o);
    const int base = __shfl_sync(FULL, myoff, o);
    if (!u) continue;
    const uint32_t lo = (uint32_t)u, hi = (uint32_t)(u >> 32);
    const int klo = base + __popc(lo & lt), khi = base + __popc(lo) + __popc(hi & lt);
    if (((lo >> lane) & 1u) && klo >= 0 && klo < kFlatItems) F.items[klo] = ((uint32_t)j << 16) | (uint32_t)lane;
    if (((hi >> lane) & 1u) && khi >= 0 && khi < kFlatItems)
      F.items[khi] = ((uint32_t)j << 16) | (uint32_t)(32 + lane);
  }
}

// X of one item and its counts: a = sx | k2 << 16, b = k3, (xlo, xhi) = its bit of X's summary
struct ItemX {
  ulonglong2 x;
  uint32_t a, b, xlo, xhi;
};
// the item's chunk of D, O, K and M
struct ItemSets {
  ulonglong2 d, o, k, m;
};
template <int CL>
__device__ __forceinline__ ItemSets flat_load(const BlkCtx& B, const FlatTabs& F, const uint16_t* wlb, Item it) {
  const int m = B.m, nw = B.nw, c = it.c;
  const uint2 inf = F.info[it.j];
  const int On = (int)(inf.x >> 16), Kn = (int)(inf.y & 0xFFFFu), Mn = (int)(inf.y >> 16);
  const int q = wlb[it.j];
  auto ptr = [&](int n) { return n >= m ? B.lab + (size_t)(n - m) * nw : B.leaf + (size_t)n * nw; };
  auto L2 = [](const uint64_t* p) { return CL == 1 ? ld2(p) : ld2_cg(p); };
  ItemSets v;
  v.d = L2(B.lab + (size_t)q * nw + 2 * c);
  v.o = L2(ptr(On) + 2 * c);
  v.k = L2(ptr(Kn) + 2 * c);
  v.m = L2(ptr(Mn) + 2 * c);
  return v;
}
__device__ __forceinline__ ItemX flat_compute(const BlkCtx& B, Item it, const ItemSets& v) {
  const int c = it.c;
  const ulonglong2 d = v.d, o = v.o, k = v.k, mm = v.m;
  ItemX r;
  r.x = make_ulonglong2((k.x | o.x) & (mm.x | d.x), (k.y | o.y) & (mm.y | d.y));
  uint64_t n0 = ~0ull, n1 = ~0ull;
  if (B.slicing) {
    n0 = ~B.S[2 * c];
    n1 = ~B.S[2 * c + 1];
  }
  const uint64_t xm0 = r.x.x & n0, xm1 = r.x.y & n1;
  const uint32_t sx = (uint32_t)(__popcll(xm0) + __popcll(xm1));
  const uint32_t k2 = (uint32_t)(__popcll(k.x & o.x & ~r.x.x & n0) + __popcll(k.y & o.y & ~r.x.y & n1));
  r.a = sx | (k2 << 16);
  r.b = (uint32_t)(__popcll(xm0 & mm.x & ~d.x) + __popcll(xm1 & mm.y & ~d.y));
  const uint32_t nz = (r.x.x | r.x.y) ? 1u : 0u;
  r.xlo = c < 32 ? nz << c : 0u;
  r.xhi = c >= 32 ? nz << (c - 32) : 0u;
  return r;
}
template <int CL>
__device__ __forceinline__ ItemX flat_eval(const BlkCtx& B, const FlatTabs& F, const uint16_t* wlb, Item it) {
  return flat_compute(B, it, flat_load<CL>(B, F, wlb, it));
}

// Add one item into its node's totals: 32-bit shared-memory atomics (lanes of one node serialise only
// among themselves; a warp-level match/reduce first measured several times slower).
__device__ __forceinline__ void flat_add(const FlatTabs& F, int j, const ItemX& v) {
  atomicAdd(&F.cnt[j].x, v.a);
  if (v.b) atomicAdd(&F.cnt[j].y, v.b);
  if (v.xlo) atomicOr(&F.xs[j].x, v.xlo);
  if (v.xhi) atomicOr(&F.xs[j].y, v.xhi);
}

__device__ __forceinline__ void flat_store(const BlkCtx& B, const FlatTabs& F, Item it, ulonglong2 x) {
  const int Pn = (int)(F.info[it.j].x & 0xFFFFu);
  *reinterpret_cast<ulonglong2*>(B.lab + (size_t)(Pn - B.m) * B.nw + 2 * it.c) = x;
}

// CL = 2: one CTA of a pair; metadata writes go to both CTAs' copies (P: the other CTA's arrays).
// IPT: items a thread has in flight at once (their loads are all issued before the first is used).
template <bool PAR, int CL, int IPT = 2>
__device__ void par_phase_flat(const BlkCtx& B, const FlatTabs& F, uint16_t* wl, uint16_t* pri, uint16_t* par,
                               int nk, uint32_t sweep, uint32_t chain, BlkCounters& cnt, const PeerArrays& P,
                               const FollowCtx* fol = nullptr) {
  const int tid = threadIdx.x, T = blockDim.x, lane = tid & 31, warp = tid >> 5, nwarps = T >> 5;
  const int m = B.m;
  const int NB = min(kFlatBatch, T);  // owners are threads 0..NB-1
  for (int b0 = 0; b0 < nk; b0 += NB) {
    const int nb = min(NB, nk - b0);
    const uint16_t* wlb = wl + b0;
    // 1. owners: rule, pivot and chunk union
    int q = 0, nck = 0;
    bool prop = false, first = true;
    uint32_t chv = 0;
    if (tid < nb) {
      q = wlb[tid];
      chv = B.ch[q];
      first = (pri[q] & 1u) != 0;  // an even priority marks a follow-up visit
      const int l = (int)(chv & 0xFFFFu), r = (int)(chv >> 16);
      const bool li = l >= m, ri = r >= m;
      prop = li || ri;
      uint2 inf = make_uint2(0xFFFFFFFFu, 0xFFFFFFFFu);
      uint64_t u = 0;
      if (prop) {
        const U4 rnd = philox10((uint32_t)(m + q), first ? sweep : follow_sweep(sweep), chain, 0u, B.key0, B.key1);
        const int rule = pick_rule(li, ri, rnd.x);
        const int slotP = rule >> 1, slotM = ((rule ^ (rule >> 1)) & 1) ^ 1;
        const int Pn = slotP ? r : l, On = slotP ? l : r;
        const uint32_t chp = B.ch[Pn - m];
        const int Mn = slotM ? (int)(chp >> 16) : (int)(chp & 0xFFFFu);
        const int Kn = slotM ? (int)(chp & 0xFFFFu) : (int)(chp >> 16);
        auto so = [&](int n) { return n >= m ? B.sum[n - m] : B.leaf_sum[n]; };
        u = B.sum[q] | so(On) | so(Kn) | so(Mn);
        nck = __popcll(u);
        inf = make_uint2((uint32_t)Pn | ((uint32_t)On << 16), (uint32_t)Kn | ((uint32_t)Mn << 16));
        F.rnd[tid] = rnd.y;
      }
      F.info[tid] = inf;
      F.u[tid] = u;
      F.cnt[tid] = make_uint2(0u, 0u);
      F.xs[tid] = make_uint2(0u, 0u);
    }
    // 2. exclusive scan of the chunk counts
    int incl = nck;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) F.scan[warp] = incl;
    __syncthreads();
    int total, before;
    {  // every warp sums the warp totals itself (no second barrier)
      const int v = lane < nwarps ? F.scan[lane] : 0;
      total = __reduce_add_sync(0xFFFFFFFFu, v);
      before = __reduce_add_sync(0xFFFFFFFFu, lane < warp ? v : 0);
    }
    if (tid < nb) F.off[tid] = (uint32_t)(incl - nck + before);
    __syncthreads();
    // 3. counts of every item, in windows of kFlatItems; a thread keeps X of its first IPT items.  A batch
    // of at most min(IPT, kFlatDirect) T items decodes each item's node and chunk directly (no list)
    Item kk[IPT];
    ulonglong2 kx[IPT];
#pragma unroll
    for (int i = 0; i < IPT; i++) {
      kk[i] = Item{-1, 0};
      kx[i] = make_ulonglong2(0ull, 0ull);
    }
    const bool direct = total <= min(IPT, kFlatDirect) * T;
    for (int w0 = 0; w0 < total; w0 += kFlatItems) {
      if (!direct) {
        if (w0) __syncthreads();  // the previous window's items are consumed
        flat_build(F, nb, w0);
        __syncthreads();
      }
      const int nwin = min(kFlatItems, total - w0);
      auto item = [&](int e) { return direct ? flat_decode(F, nb, e) : item_of(F.items[e]); };
      for (int e = tid; e < nwin; e += IPT * T) {  // IPT items: all their loads issued before any is used
        Item it[IPT];
        ItemSets sv[IPT];
#pragma unroll
        for (int i = 0; i < IPT; i++) it[i] = e + i * T < nwin ? item(e + i * T) : Item{-1, 0};
#pragma unroll
        for (int i = 0; i < IPT; i++)
          if (it[i].j >= 0) sv[i] = flat_load<CL>(B, F, wlb, it[i]);
#pragma unroll
        for (int i = 0; i < IPT; i++) {
          if (it[i].j < 0) continue;
          const ItemX r = flat_compute(B, it[i], sv[i]);
          flat_add(F, it[i].j, r);
          if (w0 == 0 && e == tid) {
            kk[i] = it[i];
            kx[i] = r.x;
          }
          cnt.busy++;
        }
      }
    }
    __syncthreads();
    // a CTA pair: the other CTA has finished this phase's scan before any metadata is rewritten in its
    // copy (the caller arrived at the cluster barrier after its own scan)
    if (CL == 2 && b0 == 0) cluster_wait();
    // 4. owners: energy, Metropolis, metadata
    if (tid < nb) {
      bool acc = false;
      if (prop) {
        const uint2 inf = F.info[tid];
        const int Pn = (int)(inf.x & 0xFFFFu), On = (int)(inf.x >> 16), Mn = (int)(inf.y >> 16);
        const uint2 pk = F.cnt[tid];
        const int sx = (int)(pk.x & 0xFFFFu), k2 = (int)(pk.x >> 16), k3 = (int)pk.y;
        const uint32_t czv = B.cz[q], czp = B.cz[Pn - m];
        const int sd = (int)(czv & 0xFFFFu), sp = (int)(czp & 0xFFFFu);
        const int cP1 = sx + k2, cV1 = sd + k3;
        const float dE =
            move_energy((int)(czp >> 16), (int)(czv >> 16), sp, sd, sx, cP1, cV1, B.sc_target, B.sc_weight, B.lse);
        acc = accept_rt(B.exp_device, B.beta, B.exptab, F.rnd[tid], dE);
        cnt.prop++;
        cnt.chunks += nck;
        if (acc) {
          cnt.acc++;
          cnt.chunks_acc += nck;
          const uint32_t chp = B.ch[Pn - m];
          const bool slotP = Pn == (int)(chv >> 16), slotM = Mn == (int)(chp >> 16);
          mset<uint32_t>(B.ch, P.ch, Pn - m,
                         slotM ? ((chp & 0xFFFFu) | ((uint32_t)On << 16)) : ((chp & 0xFFFF0000u) | (uint32_t)On));
          mset<uint32_t>(B.ch, P.ch, q,
                         slotP ? ((chv & 0xFFFF0000u) | (uint32_t)Mn) : ((chv & 0xFFFFu) | ((uint32_t)Mn << 16)));
          mset<uint32_t>(B.cz, P.cz, Pn - m, ((uint32_t)cP1 << 16) | (uint32_t)sx);
          mset<uint32_t>(B.cz, P.cz, q, ((uint32_t)cV1 << 16) | (uint32_t)sd);
          mset<uint64_t>(B.sum, P.sum, Pn - m, (uint64_t)F.xs[tid].x | ((uint64_t)F.xs[tid].y << 32));
          if (PAR) {
            if (On >= m) mset<uint16_t>(par, P.par, On - m, (uint16_t)Pn);
            if (Mn >= m) mset<uint16_t>(par, P.par, Mn - m, (uint16_t)(m + q));
          }
          if (first) follow_rearm(fol, Pn, m);  // fol is null for a CTA pair
        }
      }
      F.acc[tid] = acc;
      mset<uint16_t>(pri, P.pri, q, (uint16_t)0);
      cnt.visits++;
    }
    __syncthreads();
    // 5. X into the pivots of accepted moves: the kept items from registers, the rest recomputed
#pragma unroll
    for (int i = 0; i < IPT; i++)
      if (kk[i].j >= 0 && F.acc[kk[i].j]) flat_store(B, F, kk[i], kx[i]);
    const bool rebuild = total > kFlatItems;  // the list in shared memory is the last window's
    for (int w0 = 0; w0 < total; w0 += kFlatItems) {
      const int first = w0 == 0 ? IPT * T : 0;  // window 0's items [0, IPT T) were kept in registers
      const int nwin = min(kFlatItems, total - w0);
      if (nwin <= first) continue;  // uniform
      if (rebuild) {
        __syncthreads();
        flat_build(F, nb, w0);
        __syncthreads();
      }
      for (int e = first + tid; e < nwin; e += T) {
        const Item it = item_of(F.items[e]);
        if (F.acc[it.j]) flat_store(B, F, it, flat_eval<CL>(B, F, wlb, it).x);
      }
    }
    // The next batch rewrites the tables at once, so it waits for the stores.  After the last batch the
    // caller's next phase writes wl and the tables only behind its own scan barrier, and the stores of a
    // batch of at most IPT T items read neither (X and the items come from registers): no barrier then.
    if (b0 + NB < nk || total > IPT * T) __syncthreads();
  }
}

// GM (plan.gmeta): 1 the chain's children, cost and summary words stay in its record in global memory;
// 2 also every phase scans all nodes (no unvisited lists), visits them with G lanes each, and the
// per-node scratch (slice-move costs, model-mode costs, band depths) is the chain's 2 nint words of
// a.scratch
template <bool SUMS, int ORDER, bool MODEL, int GM>
__global__ void __launch_bounds__(512, 1) k_anneal_block(SweepArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = a.L;
  const BlockSmem Bm = BlockSmem::make(L, a.slice_moves, false, GM);
  const int tid = threadIdx.x, T = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const unsigned FULL = 0xFFFFFFFFu;
  float* s_lse = reinterpret_cast<float*>(smem);
  double* s_exp = reinterpret_cast<double*>(smem + 256);
  int* sh = reinterpret_cast<int*>(smem + 768);  // block scalars
  for (int q = tid; q < 64; q += T) {
    s_lse[q] = a.lse_tab[q];
    s_exp[q] = c_exp_tab[q];
  }
  BlkCtx B;
  B.m = L.m;
  B.nint = L.nint;
  B.nw = L.nw;
  B.nchunks = L.nw / 2;
  B.key0 = a.key0;
  B.key1 = a.key1;
  B.beta = a.beta;
  B.sc_target = a.sc_target;
  B.sc_weight = a.sc_weight;
  B.slicing = a.slicing;
  B.exp_device = a.exp_device;
  B.mode = a.mode;
  B.mp = a.mp;
  B.lse = s_lse;
  B.exptab = s_exp;
  B.leaf = a.leaf;
  B.leaf_sum = a.leaf_sum;
  B.ch = GM ? nullptr : reinterpret_cast<uint32_t*>(smem + Bm.off_ch);  // GM: set per chain
  B.cz = GM ? nullptr : reinterpret_cast<uint32_t*>(smem + Bm.off_cz);
  B.sum = GM ? nullptr : reinterpret_cast<uint64_t*>(smem + Bm.off_sum);
  B.S = reinterpret_cast<uint64_t*>(smem + Bm.off_S);
  uint32_t* cz2 = GM == 2 ? nullptr : reinterpret_cast<uint32_t*>(smem + Bm.off_cz2);  // GM 2: per chain
  uint16_t* pri = reinterpret_cast<uint16_t*>(smem + Bm.off_pri);
  uint16_t* par = reinterpret_cast<uint16_t*>(smem + Bm.off_par);
  uint16_t* wl = reinterpret_cast<uint16_t*>(smem + Bm.off_wl);
  uint16_t* Ua = GM == 2 ? nullptr : reinterpret_cast<uint16_t*>(smem + Bm.off_U);
  uint16_t* Ub = GM == 2 ? nullptr : reinterpret_cast<uint16_t*>(smem + Bm.off_U2);
  float* costs = reinterpret_cast<float*>(Ua);  // model modes: node costs, while the U lists are free (GM 2: per chain)
  const int m = L.m, nint = L.nint;
  FlatTabs F;
  F.info = reinterpret_cast<uint2*>(smem + Bm.off_ninfo);
  F.rnd = reinterpret_cast<uint32_t*>(smem + Bm.off_nrnd);
  F.cnt = reinterpret_cast<uint2*>(smem + Bm.off_ncnt);
  F.xs = reinterpret_cast<uint2*>(smem + Bm.off_nxs);
  F.acc = smem + Bm.off_nacc;
  F.off = reinterpret_cast<uint32_t*>(smem + Bm.off_noff);
  F.u = reinterpret_cast<uint64_t*>(smem + Bm.off_nu);
  F.items = reinterpret_cast<uint32_t*>(smem + Bm.off_items);
  F.scan = reinterpret_cast<int*>(smem + Bm.off_scan);
  if (Bm.off_lsum) {  // leaf chunk summaries cached in shared memory
    uint64_t* ls = reinterpret_cast<uint64_t*>(smem + Bm.off_lsum);
    for (int q = tid; q < L.m; q += T) ls[q] = a.leaf_sum[q];
    B.leaf_sum = ls;
  }
  BlkCounters cnt{};
  __syncthreads();
  for (int c = blockIdx.x; c < a.nchains; c += gridDim.x) {
    uint8_t* grec = a.recs + (size_t)c * L.rec_bytes;
    B.lab = reinterpret_cast<uint64_t*>(grec);
    const uint32_t* gch = reinterpret_cast<const uint32_t*>(grec + L.off_ch);
    const uint32_t* gcz = reinterpret_cast<const uint32_t*>(grec + L.off_cz);
    const uint64_t* gS = reinterpret_cast<const uint64_t*>(grec + L.off_S);
    if constexpr (GM != 0) {
      B.ch = reinterpret_cast<uint32_t*>(grec + L.off_ch);
      B.cz = reinterpret_cast<uint32_t*>(grec + L.off_cz);
      B.sum = reinterpret_cast<uint64_t*>(grec + L.off_sum);
      if constexpr (GM == 2) {
        cz2 = a.scratch ? a.scratch + (size_t)c * 2 * nint : nullptr;
        costs = a.scratch ? reinterpret_cast<float*>(cz2 + nint) : nullptr;
      }
    } else {
      for (int q = tid; q < nint; q += T) {
        B.ch[q] = gch[q];
        B.cz[q] = gcz[q];
      }
      if (SUMS) {
        const uint64_t* gs = reinterpret_cast<const uint64_t*>(grec + L.off_sum);
        for (int q = tid; q < nint; q += T) B.sum[q] = gs[q];
      }
    }
    for (int q = tid; q < L.nw; q += T) B.S[q] = gS[q];
    __syncthreads();
    const uint32_t chain = (uint32_t)(a.chain0 + c);
    const uint32_t hc = chain_hash(chain, a.key0);
    if (ORDER == 0) {
      for (int q = tid; q < nint; q += T) {
        uint32_t cw = B.ch[q];
        int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
        if (l >= m) par[l - m] = (uint16_t)(m + q);
        if (r >= m) par[r - m] = (uint16_t)(m + q);
      }
      if (tid == 0) par[nint - 1] = 0xFFFFu;
      __syncthreads();
    }
    for (int s = 0; s < a.nsweeps; s++) {
      const uint32_t sw = a.sweep0 + (uint32_t)s;
      if (ORDER == 0) {
        const uint32_t hs = sweep_hash(sw, hc);
        if (a.par_band > 0) {
          // depths at the start of the sweep in (pri, wl) and (U, U2) read as word arrays (GM 2: in the
          // chain's scratch words)
          uint32_t* A0 = GM == 2 ? cz2 : reinterpret_cast<uint32_t*>(pri);
          uint32_t* U32 = GM == 2 ? cz2 + nint : reinterpret_cast<uint32_t*>(Ua);
          block_depths(par, m, nint, A0, U32);
          for (int q = tid; q < nint; q += T)
            pri[q] = (uint16_t)band_pri(node_pri((uint32_t)(m + q), hs), (int)(U32[q] >> 16), a.par_band);
          __syncthreads();
          if (GM != 2)
            for (int q = tid; q < nint; q += T) Ua[q] = (uint16_t)q;
        } else {
          for (int q = tid; q < nint; q += T) {
            pri[q] = (uint16_t)node_pri((uint32_t)(m + q), hs);
            if (GM != 2) Ua[q] = (uint16_t)q;
          }
        }
        uint16_t *U = Ua, *U2 = Ub;
        int nU = nint;
        const bool follow = a.par_follow != 0;
        const int max_phases = follow ? 2 * nint : nint;
        // the scan counters alternate between sh[0..1] (even phases) and sh[2..3] (odd phases): a phase
        // clears the next phase's pair behind its own scan barrier, so no barrier is spent on clearing
        if (tid == 0) sh[0] = sh[1] = sh[2] = sh[3] = 0;
        __syncthreads();
        for (int guard = 0; guard <= max_phases; guard++) {
          int* const ctr = sh + 2 * (guard & 1);
          if constexpr (GM == 2)
            phase_scan<4, false>(nullptr, nint, wl, nullptr, ctr, pri, par, B.ch, m);
          else
            phase_scan<4>(U, nU, wl, U2, ctr, pri, par, B.ch, m);
          __syncthreads();
          const int nk = ctr[0];
          nU = ctr[1];
          if (tid == 0) sh[2 * ((guard + 1) & 1)] = sh[2 * ((guard + 1) & 1) + 1] = 0;
          uint16_t* tmp = U;
          U = U2;
          U2 = tmp;
          if (nk == 0) break;
          if (tid == 0) cnt.steps++;
          // re-armed pivots (par_follow) are appended to U after the nU kept nodes, counted on in ctr[1]
          const FollowCtx fctx{pri, GM == 2 ? nullptr : U, &ctr[1], hs};
          const FollowCtx* fol = follow ? &fctx : nullptr;
          if constexpr (SUMS && !MODEL && GM != 2) {
            par_phase_flat<true, 1>(B, F, wl, pri, par, nk, sw, chain, cnt, PeerArrays{}, fol);
          } else {
            const int G = pick_group(nk, T);
            const int groups = T / G, g = tid / G, t = tid & (G - 1);
            const unsigned gm = G == 32 ? FULL : (((1u << G) - 1u) << (lane & ~(G - 1)));
            for (int j = g; j < nk; j += groups) {
              int q = wl[j];
              const bool first = (pri[q] & 1u) != 0;  // an even priority marks a follow-up visit
              visit_coop<SUMS, true, MODEL>(B, par, m + q, first ? sw : follow_sweep(sw), chain, G, t, gm, cnt,
                                            first ? fol : nullptr);
              if (t == 0) {
                pri[q] = 0;
                cnt.visits++;
              }
              cnt.busy++;
            }
            __syncthreads();
          }
          if (follow) nU = ctr[1];  // cleared again only behind the next phase's scan barrier
        }
      } else {
        if (tid == 0) {
          wl[0] = (uint16_t)(nint - 1);
          sh[2] = 1;
        }
        __syncthreads();
        for (int guard = 0; guard <= nint; guard++) {
          const int sp = sh[2];
          if (sp <= 0) break;
          const int G = pick_group(min(sp, T), T);
          const int groups = T / G, g = tid / G, t = tid & (G - 1);
          const unsigned gm = G == 32 ? FULL : (((1u << G) - 1u) << (lane & ~(G - 1)));
          const int k = min(sp, groups), b0 = sp - k;
          const int q = g < k ? (int)wl[b0 + g] : 0;
          __syncthreads();
          if (tid == 0) {
            sh[2] = b0;
            cnt.steps++;
          }
          __syncthreads();
          if (g < k) {
            visit_coop<SUMS, false, MODEL>(B, par, m + q, sw, chain, G, t, gm, cnt);
            if (t == 0) {
              cnt.visits++;
              uint32_t cw = B.ch[q];
              int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
              int n = (l >= m) + (r >= m);
              if (n) {
                int pos = atomicAdd(&sh[2], n);
                if (r >= m) wl[pos++] = (uint16_t)(r - m);
                if (l >= m) wl[pos] = (uint16_t)(l - m);
              }
            }
            cnt.busy++;
          }
          __syncthreads();
        }
      }
      if (a.slice_moves > 0 && (sw + 1) % (uint32_t)a.slice_every == 0) {
        __syncthreads();
        slice_step_block(B, a, cz2, sh + 8, nullptr, sw, chain, cnt, MODEL ? costs : nullptr);
      }
      __syncthreads();
    }
    if (MODEL) block_model_costs(B, costs);
    if (warp == 0) {
      EvalOut e = eval_cz(B.cz, nint, B.S, L.nw, B.leaf, m, B.slicing, a.leaf_sc, lane, MODEL ? costs : nullptr);
      if (lane == 0) {
        a.out_lc[c] = e.lcost;
        a.out_sc[c] = e.sc;
        a.out_ns[c] = e.ns;
      }
    }
    uint32_t* wch = reinterpret_cast<uint32_t*>(grec + L.off_ch);
    uint32_t* wcz = reinterpret_cast<uint32_t*>(grec + L.off_cz);
    uint64_t* wS = reinterpret_cast<uint64_t*>(grec + L.off_S);
    if constexpr (GM == 0) {
      for (int q = tid; q < nint; q += T) {
        wch[q] = B.ch[q];
        wcz[q] = B.cz[q];
      }
      if (SUMS) {
        uint64_t* ws = reinterpret_cast<uint64_t*>(grec + L.off_sum);
        for (int q = tid; q < nint; q += T) ws[q] = B.sum[q];
      }
    }
    for (int q = tid; q < L.nw; q += T) wS[q] = B.S[q];
    cnt.flush(a.stats, 32);  // slice moves were counted by all 32 lanes of warp 0
    __syncthreads();
  }
}

// ================================================================================================
// k_anneal_cluster: par order with chunk summaries, one chain per cluster of two CTAs on two SMs.
// With fewer chains than SMs (the 64x64 lattice runs 72 chains on 148 SMs) a CTA per chain leaves half of
// the GPU idle; here both CTAs of a pair hold a full copy of the chain's per-node metadata in their own
// shared memory, and every metadata write of a visit goes to both copies (a distributed-shared-memory
// store).  CTA r owns the nodes q with q % 2 == r: it scans them for the phase's independent set and
// visits the active ones with par_phase_flat; label sets stay in HBM (loaded L2-only).  Per phase the
// two CTAs meet at a split cluster barrier (each arrives after its scan and waits before its first store
// into the other's copy, so no scan reads a word the phase rewrites) and at a full one at the end, which
// also exchanges their active counts; the phase sequence and every move are those of k_anneal_block,
// so the chains are bit-identical.
// ================================================================================================
__global__ void __launch_bounds__(512, 1) k_anneal_cluster(SweepArgs a) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const Layout L = a.L;
  const BlockSmem Bm = BlockSmem::make(L, a.slice_moves, true);
  const int tid = threadIdx.x, T = blockDim.x, lane = tid & 31;
  const unsigned FULL = 0xFFFFFFFFu;
  float* s_lse = reinterpret_cast<float*>(smem);
  double* s_exp = reinterpret_cast<double*>(smem + 256);
  int* sh = reinterpret_cast<int*>(smem + 768);  // [0,4) scan counters (a pair per phase parity), [4,6) the peer's active counts
  for (int q = tid; q < 64; q += T) {
    s_lse[q] = a.lse_tab[q];
    s_exp[q] = c_exp_tab[q];
  }
  BlkCtx B;
  B.m = L.m;
  B.nint = L.nint;
  B.nw = L.nw;
  B.nchunks = L.nw / 2;
  B.key0 = a.key0;
  B.key1 = a.key1;
  B.beta = a.beta;
  B.sc_target = a.sc_target;
  B.sc_weight = a.sc_weight;
  B.slicing = a.slicing;
  B.exp_device = a.exp_device;
  B.mode = 0;  // tc only (the plan)
  B.lse = s_lse;
  B.exptab = s_exp;
  B.leaf = a.leaf;
  B.leaf_sum = a.leaf_sum;
  B.ch = reinterpret_cast<uint32_t*>(smem + Bm.off_ch);
  B.cz = reinterpret_cast<uint32_t*>(smem + Bm.off_cz);
  B.sum = reinterpret_cast<uint64_t*>(smem + Bm.off_sum);
  B.S = reinterpret_cast<uint64_t*>(smem + Bm.off_S);
  uint32_t* cz2 = reinterpret_cast<uint32_t*>(smem + Bm.off_cz2);
  uint16_t* pri = reinterpret_cast<uint16_t*>(smem + Bm.off_pri);
  uint16_t* par = reinterpret_cast<uint16_t*>(smem + Bm.off_par);
  uint16_t* wl = reinterpret_cast<uint16_t*>(smem + Bm.off_wl);
  uint16_t* Ua = reinterpret_cast<uint16_t*>(smem + Bm.off_U);
  uint16_t* Ub = reinterpret_cast<uint16_t*>(smem + Bm.off_U2);
  const int m = L.m, nint = L.nint;
  FlatTabs F;
  F.info = reinterpret_cast<uint2*>(smem + Bm.off_ninfo);
  F.rnd = reinterpret_cast<uint32_t*>(smem + Bm.off_nrnd);
  F.cnt = reinterpret_cast<uint2*>(smem + Bm.off_ncnt);
  F.xs = reinterpret_cast<uint2*>(smem + Bm.off_nxs);
  F.acc = smem + Bm.off_nacc;
  F.off = reinterpret_cast<uint32_t*>(smem + Bm.off_noff);
  F.u = reinterpret_cast<uint64_t*>(smem + Bm.off_nu);
  F.items = reinterpret_cast<uint32_t*>(smem + Bm.off_items);
  F.scan = reinterpret_cast<int*>(smem + Bm.off_scan);
  if (Bm.off_lsum) {  // leaf chunk summaries cached in shared memory
    uint64_t* ls = reinterpret_cast<uint64_t*>(smem + Bm.off_lsum);
    for (int q = tid; q < L.m; q += T) ls[q] = a.leaf_sum[q];
    B.leaf_sum = ls;
  }
  // the other CTA's array bases live in this CTA's block scalars (bytes 64..103 of that area), read when a
  // decision writes both copies, so that they hold no registers through the rest of a phase
  PeerArrays& P = *reinterpret_cast<PeerArrays*>(smem + 768 + 64);
  if (tid == 0) {
    P.ch = cl.map_shared_rank(B.ch, rank ^ 1);
    P.cz = cl.map_shared_rank(B.cz, rank ^ 1);
    P.sum = cl.map_shared_rank(B.sum, rank ^ 1);
    P.par = cl.map_shared_rank(par, rank ^ 1);
    P.pri = cl.map_shared_rank(pri, rank ^ 1);
  }
  int* peer_sh = cl.map_shared_rank(sh, rank ^ 1);
  BlkCounters cnt{};
  const int npair = (int)(gridDim.x / 2);
  for (int c = (int)(blockIdx.x / 2); c < a.nchains; c += npair) {
    uint8_t* grec = a.recs + (size_t)c * L.rec_bytes;
    B.lab = reinterpret_cast<uint64_t*>(grec);
    const uint32_t* gch = reinterpret_cast<const uint32_t*>(grec + L.off_ch);
    const uint32_t* gcz = reinterpret_cast<const uint32_t*>(grec + L.off_cz);
    const uint64_t* gS = reinterpret_cast<const uint64_t*>(grec + L.off_S);
    const uint64_t* gs = reinterpret_cast<const uint64_t*>(grec + L.off_sum);
    for (int q = tid; q < nint; q += T) {
      const uint32_t cw = gch[q];
      B.ch[q] = cw;
      B.cz[q] = gcz[q];
      B.sum[q] = gs[q];
      const int l = (int)(cw & 0xFFFFu), r = (int)(cw >> 16);
      if (l >= m) par[l - m] = (uint16_t)(m + q);
      if (r >= m) par[r - m] = (uint16_t)(m + q);
    }
    if (tid == 0) par[nint - 1] = 0xFFFFu;
    for (int q = tid; q < L.nw; q += T) B.S[q] = gS[q];
    __syncthreads();  // the copy is complete before any thread reads it (par_band reads par first)
    const uint32_t chain = (uint32_t)(a.chain0 + c);
    const uint32_t hc = chain_hash(chain, a.key0);
    int ph = 0;  // phases of this chain: parity selects the exchange slot
    for (int s = 0; s < a.nsweeps; s++) {
      const uint32_t sw = a.sweep0 + (uint32_t)s;
      const uint32_t hs = sweep_hash(sw, hc);
      if (a.par_band > 0) {  // both CTAs compute the same depths from their identical copies
        uint32_t* U32 = reinterpret_cast<uint32_t*>(Ua);
        block_depths(par, m, nint, reinterpret_cast<uint32_t*>(pri), U32);
        for (int q = tid; q < nint; q += T)
          pri[q] = (uint16_t)band_pri(node_pri((uint32_t)(m + q), hs), (int)(U32[q] >> 16), a.par_band);
        __syncthreads();
      } else {
        for (int q = tid; q < nint; q += T) pri[q] = (uint16_t)node_pri((uint32_t)(m + q), hs);
      }
      int nU = (nint - rank + 1) / 2;  // the nodes q = 2j + rank
      for (int j = tid; j < nU; j += T) Ua[j] = (uint16_t)(2 * j + rank);
      uint16_t *U = Ua, *U2 = Ub;
      // scan counters alternate between sh[0..1] and sh[2..3] by phase (cleared behind the scan barrier)
      if (tid == 0) sh[0] = sh[1] = sh[2] = sh[3] = 0;
      // both copies are complete (loaded or initialised) before either CTA writes into the other
      cl.sync();
      for (int guard = 0; guard <= nint; guard++, ph++) {
        int* const ctr = sh + 2 * (guard & 1);
        phase_scan<4>(U, nU, wl, U2, ctr, pri, par, B.ch, m);
        __syncthreads();
        const int nk = ctr[0];
        nU = ctr[1];
        if (tid == 0) sh[2 * ((guard + 1) & 1)] = sh[2 * ((guard + 1) & 1) + 1] = 0;
        uint16_t* tmp = U;
        U = U2;
        U2 = tmp;
        // this CTA's scan is done: the other CTA may rewrite this copy's metadata once it has waited
        cluster_arrive();
        if (nk > 0)
          par_phase_flat<true, 2>(B, F, wl, pri, par, nk, sw, chain, cnt, P);  // waits before its writes
        else
          cluster_wait();
        if (tid == 0) peer_sh[4 + (ph & 1)] = nk;
        cl.sync();
        const int total = nk + sh[4 + (ph & 1)];
        if (total == 0) break;
        if (tid == 0 && rank == 0) cnt.steps++;
      }
      if (a.slice_moves > 0 && (sw + 1) % (uint32_t)a.slice_every == 0) {
        // both CTAs make the same slice moves on their own copies (same data, same random numbers)
        __syncthreads();
        slice_step_block(B, a, cz2, sh + 8, nullptr, sw, chain, cnt);
      }
      __syncthreads();
    }
    if (rank == 0) {
      if (tid < 32) {
        EvalOut e = eval_cz(B.cz, nint, B.S, L.nw, B.leaf, m, B.slicing, a.leaf_sc, lane);
        if (lane == 0) {
          a.out_lc[c] = e.lcost;
          a.out_sc[c] = e.sc;
          a.out_ns[c] = e.ns;
        }
      }
      uint32_t* wch = reinterpret_cast<uint32_t*>(grec + L.off_ch);
      uint32_t* wcz = reinterpret_cast<uint32_t*>(grec + L.off_cz);
      uint64_t* wS = reinterpret_cast<uint64_t*>(grec + L.off_S);
      uint64_t* ws = reinterpret_cast<uint64_t*>(grec + L.off_sum);
      for (int q = tid; q < nint; q += T) {
        wch[q] = B.ch[q];
        wcz[q] = B.cz[q];
        ws[q] = B.sum[q];
      }
      for (int q = tid; q < L.nw; q += T) wS[q] = B.S[q];
    }
    cnt.flush(a.stats, rank == 0 ? 32 : 0);  // slice moves: all 32 lanes of warp 0 of both CTAs
    __syncthreads();
  }
  // the peer may still write into this CTA's shared memory until both have left the last phase
  cl.sync();
}

// Population resampling: dst chain c <- src chain anc[c] (reference k_copy, :1017-1022).
__global__ void k_copy(const uint4* __restrict__ src, uint4* __restrict__ dst, const int* __restrict__ anc, int n4) {
  const uint4* s = src + (size_t)anc[blockIdx.x] * n4;
  uint4* d = dst + (size_t)blockIdx.x * n4;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d[i] = s[i];
}
// The same gather from two sources: record k of [a (na records) ++ b] (a multi-GPU resampling step: the
// rank's own records, then the ones it received), without first copying a and b into one buffer.
__global__ void k_copy2(const uint4* __restrict__ a, int na, const uint4* __restrict__ b, uint4* __restrict__ dst,
                        const int* __restrict__ idx, int n4) {
  const int k = idx[blockIdx.x];
  const uint4* s = k < na ? a + (size_t)k * n4 : b + (size_t)(k - na) * n4;
  uint4* d = dst + (size_t)blockIdx.x * n4;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d[i] = s[i];
}

// ------------------------------------------------------------------------------------------------
// Host side: plans and launches
// ------------------------------------------------------------------------------------------------
template <int NW, int ORDER>
static cudaError_t launch_warp_t(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  auto k = a.mode != 0 ? k_anneal_warp<NW, ORDER, true> : k_anneal_warp<NW, ORDER, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  k<<<p.grid, 32 * p.warps_per_cta, p.smem, st>>>(a, p.warps_per_cta);
  return cudaGetLastError();
}

template <int NW>
static cudaError_t launch_pair_t(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  auto k = k_anneal_pair<NW>;
  size_t smem = PairSmem::make(a.L, p.warps_per_cta, a.slice_moves).total;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<p.grid, 64 * p.warps_per_cta, smem, st>>>(a, p.warps_per_cta);
  return cudaGetLastError();
}

static cudaError_t launch_pair(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  switch (a.L.nw) {
    case 1: return launch_pair_t<1>(a, p, st);
    case 2: return launch_pair_t<2>(a, p, st);
    case 4: return launch_pair_t<4>(a, p, st);
    case 6: return launch_pair_t<6>(a, p, st);
    case 8: return launch_pair_t<8>(a, p, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int ORDER>
// ORDER: 0 par, 1 pre-order, 2 par with par_band / par_follow
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

template <bool SUMS, int ORDER>
static cudaError_t launch_block_t(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  auto k = p.gmeta == 2 ? (a.mode != 0 ? k_anneal_block<SUMS, ORDER, true, 2> : k_anneal_block<SUMS, ORDER, false, 2>)
            : p.gmeta   ? (a.mode != 0 ? k_anneal_block<SUMS, ORDER, true, 1> : k_anneal_block<SUMS, ORDER, false, 1>)
                        : (a.mode != 0 ? k_anneal_block<SUMS, ORDER, true, 0> : k_anneal_block<SUMS, ORDER, false, 0>);
  if (p.gmeta == 2 && !a.scratch && (a.slice_moves > 0 || a.mode != 0 || a.par_band > 0)) return cudaErrorInvalidValue;
  size_t smem = BlockSmem::make(a.L, a.slice_moves, false, p.gmeta).total;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<p.grid, 32 * p.warps_per_cta, smem, st>>>(a);
  return cudaGetLastError();
}

static cudaLaunchConfig_t cluster_config(int grid, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(512, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

static cudaError_t launch_cluster(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  size_t smem = BlockSmem::make(a.L, a.slice_moves, true).total;
  cudaError_t e = cudaFuncSetAttribute(k_anneal_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cluster_config(p.grid, smem, st, attr);
  return cudaLaunchKernelEx(&cfg, k_anneal_cluster, a);
}

// Chains that a CTA-pair launch keeps resident at once (0 if the pair cannot be launched).
static int cluster_capacity(size_t smem, int grid) {
  if (cudaFuncSetAttribute(k_anneal_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 0;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cluster_config(grid, smem, 0, attr);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k_anneal_cluster, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

cudaError_t plan_sweeps(const Layout& L, int nchains, int device, int hint, int order, int slice_moves, int par_band,
                        int par_follow, int model, LaunchPlan* plan) {
  int nsm = 0, optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) return e;
  bool warp_ok = (L.nw == 1 || L.nw == 2 || L.nw == 4 || L.nw == 6 || L.nw == 8) && hint != 2;
  // par order: two warps per chain (up to 14 pairs per SM; plain par order only)
  if (warp_ok && order == 0 && hint == 3) {
    int np = 14;
    while (np > 0 && PairSmem::make(L, np, slice_moves).total > (uint32_t)optin) np--;
    if (np > 0) {
      int need = (nchains + np - 1) / np;
      while (np > 1 && need < nsm) {
        np = (np + 1) / 2;
        need = (nchains + np - 1) / np;
      }
      plan->kind = K_PAIR;
      plan->warps_per_cta = np;
      plan->grid = need < nsm ? need : nsm;
      plan->smem = PairSmem::make(L, np, slice_moves).total;
      return cudaSuccess;
    }
  }
  if (hint == 3) return cudaErrorNotSupported;
  if (warp_ok) {
    // as many chain slots per CTA as fit (at most 16 warps), one CTA per SM
    int wpc = 16;
    while (wpc > 0 && WarpSmem::make(L, wpc, slice_moves).total > (uint32_t)optin) wpc--;
    if (wpc > 0) {
      // Chains run in waves of nsm * wpc; every chain of a launch does the same number of sweeps, so the
      // launch takes (number of waves) chain times.  Use the fewest warps per CTA that keep that number
      // of waves: no slot idles in the last wave, and fewer warps share each SM's issue slots.
      const long slots = (long)nsm * wpc;
      const long waves = (nchains + slots - 1) / slots;
      wpc = (int)((nchains + (long)nsm * waves - 1) / ((long)nsm * waves));
      const int need = (nchains + wpc - 1) / wpc;
      plan->kind = K_WARP;
      plan->warps_per_cta = wpc;
      plan->grid = need < nsm ? need : nsm;
      plan->smem = WarpSmem::make(L, wpc, slice_moves).total;
      return cudaSuccess;
    }
  }
  // one CTA per chain, label sets in HBM: 16 warps, or 8 when two CTAs fit on an SM and the chains fill
  // more than one wave
  if (hint == 1) return cudaErrorNotSupported;
  BlockSmem bs = BlockSmem::make(L, slice_moves);
  plan->gmeta = 0;
  if (bs.total > (uint32_t)optin) {
    // the per-node metadata does not fit: keep children, cost and summary words in the record
    bs = BlockSmem::make(L, slice_moves, false, 1);
    plan->gmeta = 1;
    if (bs.total > (uint32_t)optin) {
      // the largest networks: 6 bytes a node in shared memory, every phase scans all nodes
      bs = BlockSmem::make(L, slice_moves, false, 2);
      if (bs.total > (uint32_t)optin) return cudaErrorNotSupported;
      plan->gmeta = 2;
    }
  }
  plan->kind = K_BLOCK;
  plan->warps_per_cta = 16;
  plan->grid = nchains;
  {
    // more chains than SMs: two CTAs of 8 warps per SM where both fit, so that one chain's barrier and L2
    // waits overlap the other chain's work (C5: 4.8e9 visits/s against 3.8e9 with one 16-warp CTA per
    // SM; four 4-warp CTAs measured 2.5e9).  Registers fit: launch bounds cap a thread at 128.
    int smem_sm = 0;
    e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
    if (e != cudaSuccess) return e;
    if (nchains > nsm && 2u * (bs.total + 1024u) <= (uint32_t)smem_sm) plan->warps_per_cta = 8;
  }
  plan->smem = bs.total;
  plan->cluster = 1;
  // par order with chunk summaries and at most half as many chains as SMs: a pair of CTAs per chain,
  // if every pair can be resident at once
  const bool pair_ok = L.sums && order == 0 && slice_moves == 0 && !par_follow && !model && !plan->gmeta;
  if (hint == 4 && !pair_ok) return cudaErrorNotSupported;
  if (pair_ok && (hint == 4 || (hint == 0 && 2 * nchains <= nsm))) {
    const int grid = 2 * nchains;
    const uint32_t psmem = BlockSmem::make(L, slice_moves, true).total;
    if (psmem <= (uint32_t)optin && cluster_capacity(psmem, grid) >= (hint == 4 ? 1 : nchains)) {
      plan->grid = grid;
      plan->cluster = 2;
      plan->smem = psmem;
    } else if (hint == 4) {
      return cudaErrorNotSupported;
    }
  }
  return cudaSuccess;
}

cudaError_t launch_sweeps(const SweepArgs& a, const LaunchPlan& p, cudaStream_t st) {
  if (p.kind == K_PAIR) return launch_pair(a, p, st);
  if (p.kind == K_WARP) {
    if (a.order != 0) return launch_warp_o<1>(a, p, st);
    return a.par_band || a.par_follow ? launch_warp_o<2>(a, p, st) : launch_warp_o<0>(a, p, st);
  }
  if (p.cluster == 2) return launch_cluster(a, p, st);
  if (a.L.sums) return a.order == 0 ? launch_block_t<true, 0>(a, p, st) : launch_block_t<true, 1>(a, p, st);
  return a.order == 0 ? launch_block_t<false, 0>(a, p, st) : launch_block_t<false, 1>(a, p, st);
}

cudaError_t launch_copy_chains(const uint8_t* src, uint8_t* dst, const int* anc, int nchains, uint32_t rec_bytes,
                               cudaStream_t st) {
  if (nchains <= 0) return cudaSuccess;
  k_copy<<<nchains, 256, 0, st>>>(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), anc,
                                  (int)(rec_bytes / 16));
  return cudaGetLastError();
}

cudaError_t launch_copy_chains2(const uint8_t* a, int na, const uint8_t* b, uint8_t* dst, const int* idx, int nchains,
                                uint32_t rec_bytes, cudaStream_t st) {
  if (nchains <= 0) return cudaSuccess;
  k_copy2<<<nchains, 256, 0, st>>>(reinterpret_cast<const uint4*>(a), na, reinterpret_cast<const uint4*>(b),
                                   reinterpret_cast<uint4*>(dst), idx, (int)(rec_bytes / 16));
  return cudaGetLastError();
}

cudaError_t upload_lse_table(const float* host64, float* dev64, cudaStream_t st) {
  cudaError_t e = cudaMemcpyToSymbolAsync(c_exp_tab, kExp2Tab64, sizeof(kExp2Tab64), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaMemcpyAsync(dev64, host64, 64 * sizeof(float), cudaMemcpyHostToDevice, st);
}

int fixup_count() { return kExpfFixN; }

// Self-test of the Metropolis arithmetic over the float bit patterns [lo, hi] (all negative):
// checksum of the device's host-libm-equivalent expf (Tang + fix-up table) and the largest relative
// error of the ex2.approx pre-test against the correctly rounded value for x >= -17.5.
__global__ void k_expf_selftest(uint32_t lo, uint32_t hi, unsigned long long* sum, unsigned int* maxerr_bits) {
  __shared__ double T[64];
  for (int q = threadIdx.x; q < 64; q += blockDim.x) T[q] = c_exp_tab[q];
  __syncthreads();
  unsigned long long acc = 0;
  float worst = 0.f;
  const uint64_t n = (uint64_t)hi - lo + 1;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t xb = lo + (uint32_t)k;
    float x = __uint_as_float(xb);
    float e = tang_expf(x, T);
    float g = fixup_lookup(x, e, kExpfFixX, kExpfFixG, kExpfFixN);
    acc += (unsigned long long)(__float_as_uint(g) ^ (xb * 0x9E3779B1u));
    if (x >= -17.5f && e > 0.f) {
      float ea = ex2_approx(__fmul_rn(x, 1.44269504088896341f));
      float rel = fabsf(ea - e) / e;
      worst = fmaxf(worst, rel);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    worst = fmaxf(worst, __shfl_xor_sync(0xFFFFFFFFu, worst, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(sum, acc);
    atomicMax(maxerr_bits, __float_as_uint(worst));
  }
}

cudaError_t expf_selftest(uint32_t lo, uint32_t hi, unsigned long long* d_sum, unsigned int* d_err, cudaStream_t st) {
  cudaError_t e = cudaMemcpyToSymbolAsync(c_exp_tab, kExp2Tab64, sizeof(kExp2Tab64), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  k_expf_selftest<<<148 * 8, 256, 0, st>>>(lo, hi, d_sum, d_err);
  return cudaGetLastError();
}

}  // namespace tsa
