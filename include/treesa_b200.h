/* treesa_b200.h -- C ABI of the B200 TreeSA annealer (libtreesa_b200.so).
 *
 * Drop-in replacement for the reference's process boundary: treesa_gpu/driver.py:215-314 writes an
 * instance file, a tree file and a betas file, spawns the CLI binary (csrc/treesa_gpu.cu:2070-2086,
 * options parsed at :1343-1406) and reads its JSON result (:1896-1919).  Here driver.optimize fills
 * the structs below and makes one ctypes call; the result struct carries every JSON key.
 *
 * Conventions shared with the reference:
 *   - leaves are tensors 0..m-1, internal nodes m..2m-2, the root is 2m-2 (csrc/treesa_gpu.cu:15-20);
 *   - a tree is m-1 words, word i = left | right << 16 for internal node m+i (read_trees, :1077-1097);
 *   - labels are 0..nlab-1 (driver.label_map, driver.py:60-67);
 *   - chain c of the whole run (rank offset included) uses Philox counter {v, sweep, c, 0}.
 * Plain pointers and sizes only.  Every entry point returns 0 on success and a TSA_ERR_* code otherwise,
 * with a message in err; no entry point calls exit().
 */
#ifndef TREESA_B200_H
#define TREESA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSA_ABI_VERSION 2

enum {
  TSA_OK = 0,
  TSA_ERR_ARG = 1,         /* invalid instance / tree / option (reference: exit(1) in read_instance etc.) */
  TSA_ERR_INVALID = 2,     /* final tree invalid or labels mismatch (reference exit code 2, :1922) */
  TSA_ERR_CUDA = 3,        /* CUDA runtime error (reference: CK() -> exit(1), :55-62) */
  TSA_ERR_UNSUPPORTED = 4, /* option not available in this build */
  TSA_ERR_NOMEM = 5,       /* device or host allocation failed */
  TSA_ERR_TIMEOUT = 6,     /* a bounded device wait ran out (error status from a kernel) */
  TSA_ERR_COMM = 7,        /* NCCL error in a multi-GPU run */
  TSA_ERR_DEADLINE = 8     /* the run exceeded options.timeout_s (the reference driver's subprocess timeout,
                              treesa_gpu/driver.py:305) */
};

enum { TSA_MODE_TC = 0, TSA_MODE_GPU = 1, TSA_MODE_H100 = 2 };
enum { TSA_SCHEME_INDEP = 0, TSA_SCHEME_PA = 1, TSA_SCHEME_TRUNC = 2 };
enum { TSA_ORDER_PAR = 0, TSA_ORDER_PREORDER = 1 };
enum { TSA_DEBUG_ARM_ONLY = 1 };

/* Tensor network: ixs in CSR form (driver.write_instance, driver.py:70-77; read_instance,
 * csrc/treesa_gpu.cu:1035-1073).  Labels inside one tensor must be distinct. */
typedef struct tsa_instance {
  int32_t m;                  /* tensors (leaves), >= 3, 2m-1 <= 65535 */
  int32_t nlab;               /* labels 0..nlab-1 */
  const int32_t* ix_offsets;  /* [m+1] */
  const int32_t* ix_labels;   /* [ix_offsets[m]] */
  int32_t niy;                /* open (output) labels */
  const int32_t* iy;          /* [niy] */
} tsa_instance;

/* Run options: every field of the reference's Opts (csrc/treesa_gpu.cu:1279-1298) that changes the
 * result, plus placement.  Kernel-tuning options of the reference (kernel, wpb, lpc, coop_*, wpc,
 * block, chunk_sums, wide) have no counterpart: the kernel choice here never changes a result. */
typedef struct tsa_options {
  const float* betas;         /* inverse temperatures, already expanded (parse_betas, :1305-1336) */
  int32_t nbetas;
  int32_t niters;             /* sweeps per beta level */
  int32_t nchains;            /* chains of this call (this rank's shard when world_size > 1) */
  int32_t mode;               /* --mode: TSA_MODE_TC, TSA_MODE_GPU or TSA_MODE_H100 (csrc/common.h:128-222) */
  double sc_target, sc_weight;
  int32_t scheme;             /* TSA_SCHEME_* */
  double trunc_frac;
  int32_t order;              /* TSA_ORDER_* */
  uint64_t seed;
  int32_t eval_every;
  int32_t slicing;            /* 0/1 */
  int32_t slice_moves, slice_every, max_slices;
  const int32_t* init_slices; /* labels sliced initially in every chain (--init-slices) */
  int32_t ninit_slices;
  int32_t select_sc;          /* --select-sc */
  const uint32_t* init_trees; /* ntrees * (m-1) words; chain c starts from tree c % ntrees; NULL: random */
  int32_t ntrees;
  const double* gpu_model;    /* 6 values (peak_ops, bw_bits, m0, n0, k0, launch) or NULL: defaults */
  const double* h100_model;   /* 9 values (launch, perm_bw_bits, cc_bit, cc_cell, tc_bit, tc_pad_cell,
                                 tc_out_bit, small_rank, small_cell) or NULL: defaults */
  int32_t device;             /* CUDA device ordinal */
  void* stream;               /* cudaStream_t to launch on, or NULL: the library's own stream */
  int32_t rank, world_size;   /* multi-GPU: one process per GPU; chains are sharded by rank */
  const void* nccl_id;        /* 128-byte ncclUniqueId shared by all ranks (NULL when world_size == 1) */
  int32_t verbose;
  int32_t max_levels;         /* --max-levels (<= 0: all) */
  int32_t exp_mode;           /* Metropolis expf: 0 = the host libm's (bit-exact with the reference's CPU port
                                 csrc/cpu_ref.h, default); 1 = the device's expf (bit-exact with the
                                 reference's GPU binary, csrc/common.h:228 compiled by nvcc) */
  int32_t kernel_hint;        /* 0 auto; 1 one warp per chain (chain in shared memory); 2 one CTA per chain
                                 (label sets in HBM); 3 two warps per chain (par order); 4 a cluster of two
                                 CTAs per chain (par order, chunk summaries, no slice moves).  Never changes
                                 a result. */
  int32_t par_follow;         /* --par-follow (csrc/treesa_gpu.cu:1388): par order, an accepted first visit
                                 re-visits its pivot child later in the sweep if the sweep already visited it */
  int32_t par_band;           /* --par-band L (:1389): 0 off, or 2..16: par-order priorities top-down within
                                 bands of L levels of the depth at the start of each sweep */
  /* Stage 2 (--stage2-betas/--stage2-niters/--stage2-mode, :1281-1296, 1354-1357; the driver's modes
     "tc+gpu"/"tc+h100"): after the nbetas levels, continue the population on betas2 in mode2 */
  int32_t mode2;              /* TSA_MODE_GPU or TSA_MODE_H100 */
  int32_t niters2;            /* sweeps per level of stage 2 (<= 0: niters) */
  const float* betas2;        /* NULL: no stage 2 */
  int32_t nbetas2;
  float timeout_s;            /* > 0: wall-clock limit of a run's level loop, checked between levels; the run
                                 then stops with TSA_ERR_DEADLINE (single-GPU runs; 0: no limit) */
  int32_t wait_log2;          /* a bounded device wait (a chain's staging copy into shared memory) gives up
                                 after 2^wait_log2 SM cycles and the call returns TSA_ERR_TIMEOUT; 0: 31 (about
                                 a second at 1.9 GHz); 10..31 */
  int32_t debug_flags;        /* tests only, 0 otherwise.  TSA_DEBUG_ARM_ONLY: the warp kernels arm their
                                 staging barrier for a chain's record but issue no copy, so the bounded wait
                                 runs out with nothing in flight (exercises the TSA_ERR_TIMEOUT path) */
  int32_t reserved[4];
} tsa_options;

/* Result (library-owned buffers, freed by tsa_result_free).  Field names are the JSON keys of the
 * reference's output (csrc/treesa_gpu.cu:1896-1919). */
typedef struct tsa_result {
  int32_t m;
  uint32_t* tree;             /* [m-1] words left | right << 16 */
  int32_t nsliced;
  int32_t* sliced;            /* [nsliced] label ids */
  double tc, gpu_time, h100_time;   /* per slice, double precision (host_energy, :1206-1244) */
  int32_t sc;
  int32_t valid, labels_ok;
  int32_t best_chain;         /* global chain id */
  int32_t slicing, n_repair;
  double tc_total, gpu_time_total, h100_time_total;
  double t_anneal, t_init, kernel_s;
  uint64_t proposals, accepts, warp_steps, node_visits, slice_proposals, slice_accepts, busy_lanes;
  int32_t nchains, niters, nlevels, total_sweeps, W, nw, scheme, mode, nresample, order;
  int32_t ntrace;
  double* trace;              /* [ntrace][10]: t, level, beta, best_lcost_per_slice, best_sc, mean_E,
                                 families, mode, best_nsliced, mean_nsliced (:1916) */
  char kernel[32];
  uint64_t h2d_bytes, d2h_bytes;  /* host<->device bytes the call copied (inputs, energies, best chains) */
  int32_t reserved[12];
} tsa_result;

/* TSA_ABI_VERSION of the loaded library. */
int tsa_abi_version(void);
/* sizes[0..2] = sizeof(tsa_instance), sizeof(tsa_options), sizeof(tsa_result): lets a binding (ctypes,
 * cgo, ...) check its struct mirrors against this build. */
int tsa_abi_sizes(int32_t* sizes);

/* One annealing run (reference: the whole CLI run, Runner<W>::run_anneal, :1756-1923).
 * Replaces driver.py:215-314.  Thread-safe; concurrent calls on different devices run in parallel. */
int tsa_run(const tsa_instance* inst, const tsa_options* opt, tsa_result* res, char* err, size_t errlen);

/* Free the buffers of a result filled by tsa_run / tsa_session_result. */
void tsa_result_free(tsa_result* res);

/* Session API: tsa_run split into its phases, so that a caller can keep the chains resident on the
 * device and time the anneal alone (bench), or re-run it from the same initial state.
 *   create : validate, build the initial chains on the host, upload (reference: alloc + init_chains,
 *            :1564-1630)
 *   run    : every beta level: sweeps, energies, best tracking, resampling (:1789-1877)
 *   result : finalize (labels check, greedy repair, host energies; :1878-1919)
 *   reset  : restore the initial chains (device copy) and clear the run state */
typedef struct tsa_session tsa_session;
int tsa_session_create(const tsa_instance* inst, const tsa_options* opt, tsa_session** out, char* err,
                       size_t errlen);
int tsa_session_run(tsa_session* s, char* err, size_t errlen);
int tsa_session_result(tsa_session* s, tsa_result* res, char* err, size_t errlen);
int tsa_session_reset(tsa_session* s, char* err, size_t errlen);
void tsa_session_destroy(tsa_session* s);

/* Per-run counters of the last tsa_session_run (all ranks): [0] proposals, [1] accepts, [2] phases / work-
 * list steps, [3] node visits, [4] slice proposals, [5] slice accepts, [6] busy lanes, [7] sweep-kernel
 * launches (this rank), [8] 16-byte label chunks read by the proposals of the HBM kernel, [9] chunks
 * written by its accepted moves, [10] host-to-device bytes, [11] device-to-host bytes (this rank); and
 * the summed device time of the sweep kernels (this rank). */
int tsa_session_stats(tsa_session* s, uint64_t* counters12, double* kernel_seconds);

/* Where the last tsa_session_run spent its time on this rank, in seconds: t8[0] the sweep kernels, t8[1]
 * the energy gathers of runs that select level by level (population annealing, truncation, staged runs:
 * the device copy, or on several GPUs the NCCL allgather, which also waits for the slowest rank's sweeps),
 * t8[2] their population steps (the record gather, and on several GPUs the packing and the NCCL
 * send/receive of records), all three device time; t8[3] the wall time of the whole call; t8[4] host time
 * of the selection (scores, best tracking, ancestors); t8[5] wall time of fetching improved best records
 * (a copy, or an NCCL broadcast from the owner); t8[6] / t8[7] bytes of chain records this rank sent to /
 * received from other ranks in population steps.  No counterpart in the reference, which reports only
 * its kernel time (csrc/treesa_gpu.cu:1908). */
int tsa_session_timing(tsa_session* s, double* t8);

/* Population resampling of caller-held chain records (the reference's Runner::resample,
 * csrc/treesa_gpu.cu:1925-1933, and its k_copy, :1017-1022): every record c becomes a copy of record
 * anc[c], all at once.  records: device pointer to nchains records of rec_bytes bytes each (rec_bytes a
 * multiple of 16, e.g. info8[3] of a session); anc: host array of nchains ancestors in [0, nchains);
 * stream: cudaStream_t or NULL (the legacy stream) of the device that holds the records.  The gather goes
 * through a scratch copy of the population that the call allocates and frees; it returns when the
 * records hold their ancestors. */
int tsa_resample(void* records, const int32_t* anc, int32_t nchains, uint32_t rec_bytes, void* stream, char* err,
                 size_t errlen);

/* tsa_resample without any allocation, for callers that cannot allocate device memory when they
 * resample: a process whose device memory belongs to its own fixed pool, or a loop where
 * cudaMalloc/cudaFree would synchronize the device.  Same arguments and result as
 * tsa_resample; the scratch is a static device array built into the library (64 MiB of records and
 * 65536 ancestor slots, held by every GPU that loads it until exit), so at most 65536 chains and 64 MiB
 * of records; larger populations are rejected with TSA_ERR_ARG.  The first call on a device (with that
 * device current) looks the array up; make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race.  No counterpart in the reference. */
int tsa_resample_noalloc(void* records, const int32_t* anc, int32_t nchains, uint32_t rec_bytes, void* stream,
                         char* err, size_t errlen);

/* Spectral start trees (the reference's treesa_gpu/spectral.py: laplacian_vectors, path_cost).
 * tsa_laplacian_vectors: eigenvectors 2..k+1 (ascending eigenvalues) of the Laplacian of the weighted graph
 * with n vertices and the nnz unordered pairs (rows[e], cols[e], w[e]) (each pair once), as V[n][k]; dense,
 * by cuSOLVER's syevdx on the device (loaded at run time).  Replaces laplacian_vectors (spectral.py).
 * tsa_path_costs: (tc, sc) in log2 of the left-deep path tree contracting the tensors in each of the
 * norders orderings (orders[norders][m], permutations of 0..m-1).  Replaces path_cost (spectral.py). */
int tsa_laplacian_vectors(int32_t n, int32_t nnz, const int32_t* rows, const int32_t* cols, const double* w,
                          int32_t k, int32_t device, double* V, char* err, size_t errlen);
int tsa_path_costs(const tsa_instance* inst, int32_t norders, const int32_t* orders, int32_t device, double* tc,
                   int32_t* sc, char* err, size_t errlen);

/* Layout and plan of a session: info8 = {m, internal nodes, u64 words per label set, record bytes,
 * kernel (1 warp per chain, 2 CTA per chain, 3 two warps per chain, 4 two CTAs per chain, 5 CTA per
 * chain with the children/cost/summary words in global memory, 6 as 5 with every phase scanning all
 * nodes: the largest networks), warps per CTA, grid, dynamic shared memory bytes}. */
int tsa_session_info(tsa_session* s, int32_t* info8);

/* Energies of every chain after the last evaluated level (lcost per slice, sc, |S|), for tests. */
int tsa_session_energies(tsa_session* s, float* lcost, int32_t* sc, int32_t* ns, char* err, size_t errlen);

/* Copy the current chain trees ([nchains][m-1] words) and packed label sets ([nchains][m-1][nw] u64)
 * to host buffers (either may be NULL), for tests. */
int tsa_session_chains(tsa_session* s, uint32_t* trees, uint64_t* labels, char* err, size_t errlen);

/* Free the device and pinned host blocks that finished sessions left in the library's block cache
 * (kept so that repeated tsa_run calls of one workload skip the allocations; at most 8 GiB of device
 * memory and 1 GiB of pinned memory are held).  Safe to call at any time; live sessions keep theirs.
 * No counterpart in the reference, which allocates per run (csrc/treesa_gpu.cu:1565-1577). */
int tsa_release_cached_memory(void);

/* Multi-GPU rendezvous: write a fresh 128-byte ncclUniqueId into id (rank 0 calls it and shares the
 * bytes with the other ranks, e.g. through torch.distributed). */
int tsa_nccl_unique_id(void* id128, char* err, size_t errlen);

/* Transfer plan of one population-resampling step on rank `rank` of `world` (nloc chains per rank,
 * anc[g] = ancestor of global chain g): src_of[nloc] indexes [local records ++ received records];
 * send_off[world+1]/send_idx[nloc*world]: local chains sent to each rank; recv_off[world+1]/
 * recv_ids[nloc]: global chains received from each rank.  Host-only; exported for tests.
 * No counterpart in the reference (single GPU, csrc/treesa_gpu.cu:1925-1933 copies in place). */
int tsa_resample_plan(const int* anc, int nloc, int rank, int world, int* src_of, int* send_off, int* send_idx,
                      int* recv_off, int* recv_ids);

/* Self-test of the device's Metropolis arithmetic over the negative floats with bit patterns in
 * [lo_bits, hi_bits]: checksum = sum over x of (bits(expf'(x)) ^ (bits(x) * 0x9E3779B1)) mod 2^64, where
 * expf' is the device's host-libm-equivalent expf (correctly rounded Tang evaluation + fix-up table), and
 * the largest relative error of the single-instruction pre-test 2^(x log2 e) for x >= -17.5.  The host's
 * libm gives the same checksum iff the device reproduces its expf on every input of the range.
 * No counterpart in the reference (its GPU binary and its CPU port use different expf). */
int tsa_expf_selftest(int device, uint32_t lo_bits, uint32_t hi_bits, uint64_t* checksum, double* max_rel_fast,
                      char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif /* TREESA_B200_H */
