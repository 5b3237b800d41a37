// tsa_kernels.cuh -- device-side layout and launch interface of the B200 TreeSA kernels.
//
// Chain record (one per chain, in HBM, 128-byte aligned, moved whole between HBM and shared memory by
// bulk TMA copies):
//   lab[nint][nw]  u64   unsliced output-label bitset of internal node m+i (label l = bit l%64 of word
//                        l/64; nw = ceil(L/64), padded to even above 1 so a set is 16-byte aligned)
//   ch[nint]       u32   left | right << 16 (node ids: leaves 0..m-1, internal m..2m-2, root 2m-2)
//   cz[nint]       u32   cost << 16 | size of node m+i on the sliced network:
//                        size = |z & ~S|, cost = size + |x & y & ~z & ~S| (x, y: children)
//   S[nw]          u64   slice set
//   sum[nint]      u64   (wide layouts) bit c set iff 16-byte chunk c of lab[i] is nonzero
// Leaf label sets (identical for every chain) are one shared table leaf[m][nw].
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace tsa {

struct Layout {
  int m, nint, nw;           // leaves, internal nodes, u64 words per label set
  uint32_t off_ch, off_cz, off_S, rec_bytes;
  int sums;                  // 1: chunk summaries (bit c of a node's u64: 16-byte chunk c nonzero)
  uint32_t off_sum;          // summaries [nint] u64 inside the record (when sums)
};

// Everything one sweep launch needs (passed by value).
// Log-domain constants of the gpu / h100 time models (Params fields of csrc/common.h:80-93, set from
// the model dictionaries as csrc/treesa_gpu.cu:1460-1475 does).
struct ModelParams {
  float lpeak, lbw, llaunch;
  int m0, n0, k0;
  float l3launch, lperm2, lcc_bit, lcc_cell, ltc_bit, ltc_pad, ltc_out, lsmall_cell;
  int small_rank;
};

struct SweepArgs {
  Layout L;
  uint8_t* recs;             // [nchains] records of rec_bytes (input)
  uint8_t* recs_out;         // where the warp kernel writes the records back (may equal recs)
  const uint64_t* leaf;      // [m][nw]
  int nchains, chain0;       // local chain count, global id of local chain 0
  int order;                 // 0 par, 1 preorder
  float beta;
  uint32_t sweep0;
  int nsweeps;
  float sc_target, sc_weight;
  uint32_t key0, key1;
  int slicing, leaf_sc;
  int exp_device;            // 1: Metropolis with the device expf (reference GPU binary semantics)
  int slice_moves, slice_every, max_slices;
  float* out_lc;             // [nchains] per-chain energy after the launch
  int* out_sc;
  int* out_ns;
  unsigned long long* stats; // 10 device counters (see tsa_session_stats; [7] is host-side)
  int* err;                  // nonzero: a bounded wait timed out
  long long wait_cycles;     // limit of a bounded wait (SM cycles)
  int debug_arm_only;        // tests: arm the staging barrier without issuing the copy
  const float* lse_tab;      // 64 floats (device)
  const uint64_t* leaf_sum;  // [m] chunk summaries of the leaf sets (when L.sums)
  int par_band;              // par order: 0, or L = 2..16 (priorities by depth band)
  int par_follow;            // par order: re-visit the pivot child of an accepted first visit
  int mode;                  // energy of this launch: 0 tc, 1 gpu model, 2 h100 model
  ModelParams mp;
  uint32_t* scratch;         // plan gmeta 2: [nchains][2 nint] words: slice-move and model-mode costs, band depths
};

// Kernel family chosen by the host for a layout.
enum KernelKind { K_WARP = 0, K_BLOCK = 1, K_PAIR = 2 };

struct LaunchPlan {
  KernelKind kind;
  int warps_per_cta;         // chains per CTA (K_WARP), warps per chain (K_BLOCK), chain pairs (K_PAIR)
  int grid;
  size_t smem;
  int cluster = 1;           // K_BLOCK: CTAs per chain (2: k_anneal_cluster)
  int gmeta = 0;             // K_BLOCK: 1 children, cost and summary words stay in the record in global
                             // memory; 2 also no unvisited lists (every phase scans all nodes) and the
                             // slice-move cost scratch in global memory (the largest networks)
};

// Host-side entry points (tsa_kernels.cu).
// hint: 0 auto, 1 one warp per chain, 2 one CTA per chain (label sets in HBM), 3 two warps per chain,
// 4 a pair of CTAs per chain (par order with chunk summaries, no slice moves)
// model: some level of the run uses an energy mode other than tc
cudaError_t plan_sweeps(const Layout& L, int nchains, int device, int hint, int order, int slice_moves, int par_band,
                        int par_follow, int model, LaunchPlan* plan);
cudaError_t launch_sweeps(const SweepArgs& a, const LaunchPlan& plan, cudaStream_t st);
cudaError_t launch_copy_chains(const uint8_t* src, uint8_t* dst, const int* anc, int nchains, uint32_t rec_bytes,
                               cudaStream_t st);
// dst record c <- record idx[c] of [a (na records) ++ b]
cudaError_t launch_copy_chains2(const uint8_t* a, int na, const uint8_t* b, uint8_t* dst, const int* idx, int nchains,
                                uint32_t rec_bytes, cudaStream_t st);
cudaError_t upload_lse_table(const float* host64, float* dev64, cudaStream_t st);
int fixup_count();
cudaError_t expf_selftest(uint32_t lo, uint32_t hi, unsigned long long* d_sum, unsigned int* d_err, cudaStream_t st);

}  // namespace tsa
