// tsa_comm.h -- multi-GPU layer of libtreesa_b200.so: one process per GPU, chains sharded by rank
// (rank r owns global chains [r*n, (r+1)*n)).  NCCL (loaded with dlopen, so single-GPU use needs no
// NCCL) carries the only exchanges the annealer has:
//   * population schemes: allgather of every chain's (lcost, sc, |S|) after an evaluated level, so that
//     every rank computes the same resampling ancestors, and broadcast of the best chain's record from
//     its owner when the best improves;
//   * best-of-N: every rank scores its own chains level by level; one allgather of the per-level
//     summaries and of each rank's best at the end, then a broadcast of the winner's record;
//   * population resampling: chains whose ancestor lives on another rank are sent once per (source,
//     destination rank) pair with grouped ncclSend/ncclRecv into the receiver's own staging buffer,
//     then every rank gathers its new population locally.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace tsa {

struct CommImpl;

struct Comm {
  CommImpl* p = nullptr;
  int rank = 0, world = 1;
  ~Comm();
  // enqueue on st (no synchronization): every chain's energies into host buffers (pinned for overlap)
  int allgather_energies(const float* d_lc, const int* d_sc, const int* d_ns, int nloc, float* glc, int* gsc, int* gns,
                         cudaStream_t st, char* err, size_t errlen);
  // enqueue on st: the owner's record broadcast to every rank, then copied to host_out
  int fetch_record(const uint8_t* d_rec_local, uint32_t bytes, int owner, uint8_t* host_out, cudaStream_t st,
                   char* err, size_t errlen);
  int resample(const int* anc_global, uint8_t* d_rec, uint8_t* d_rec2, int* d_anc, int nloc, uint32_t rec_bytes,
               cudaStream_t st, char* err, size_t errlen);
  int sum_u64(uint64_t* host_vals, int n, cudaStream_t st, char* err, size_t errlen);
  // record bytes this rank has sent to / received from other ranks in population steps
  uint64_t sent_bytes = 0, recv_bytes = 0;
  // synchronous: n doubles from every rank, in rank order, into host_out[world*n]
  int allgather_host(const double* host_in, int n, double* host_out, cudaStream_t st, char* err, size_t errlen);
  // synchronous: the owner's host buffer copied into every rank's host buffer
  int bcast_host(uint8_t* host, uint32_t bytes, int owner, cudaStream_t st, char* err, size_t errlen);
};

int comm_create(const void* id128, int rank, int world, int device, Comm** out, char* err, size_t errlen);
int comm_unique_id(void* id128, char* err, size_t errlen);

// Host-side transfer plan of one resampling step (pure function, shared by all ranks).
//   anc[g]: ancestor (global id) of global chain g; nloc chains per rank.
//   src_of[c]: for local destination c, an index into [local records 0..nloc) ++ [received records].
//   send[q]: local chain indices this rank sends to rank q (sorted, unique).
//   recv[q]: global chain ids this rank receives from rank q (sorted, unique); received records are
//            stored in rank order, then in the order of recv[q].
struct ResamplePlan {
  int* src_of;    // [nloc]
  int* send_off;  // [world+1] offsets into send_idx
  int* send_idx;  // [<= nloc*world]
  int* recv_off;  // [world+1] offsets into recv_ids
  int* recv_ids;  // [<= nloc]
};

}  // namespace tsa

extern "C" {
// Compute the plan of rank `rank` (buffers sized as documented in ResamplePlan).  Exported for tests.
int tsa_resample_plan(const int* anc, int nloc, int rank, int world, int* src_of, int* send_off, int* send_idx,
                      int* recv_off, int* recv_ids);
}
