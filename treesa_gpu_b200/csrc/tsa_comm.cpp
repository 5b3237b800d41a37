// tsa_comm.cpp -- NCCL exchanges of the multi-GPU annealer (see tsa_comm.h).
#include "tsa_comm.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

#include "../../include/treesa_b200.h"
#include "tsa_kernels.cuh"

namespace tsa {
namespace {

void cerr_set(char* err, size_t n, const char* fmt, ...) {
  if (!err || !n) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, n, fmt, ap);
  va_end(ap);
}

// NCCL entry points resolved at run time (the library loaded by the process, e.g. torch's, is reused).
struct Nccl {
  void* h = nullptr;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) groupStart = nullptr;
  decltype(&ncclGroupEnd) groupEnd = nullptr;
  decltype(&ncclGetErrorString) errStr = nullptr;
};

const Nccl* nccl(char* err, size_t errlen) {
  static std::once_flag once;
  static Nccl N;
  static bool ok = false;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    N.h = h;
#define TSA_SYM(f, name) N.f = reinterpret_cast<decltype(N.f)>(dlsym(h, name))
    TSA_SYM(getUniqueId, "ncclGetUniqueId");
    TSA_SYM(commInitRank, "ncclCommInitRank");
    TSA_SYM(commDestroy, "ncclCommDestroy");
    TSA_SYM(allGather, "ncclAllGather");
    TSA_SYM(allReduce, "ncclAllReduce");
    TSA_SYM(broadcast, "ncclBroadcast");
    TSA_SYM(send, "ncclSend");
    TSA_SYM(recv, "ncclRecv");
    TSA_SYM(groupStart, "ncclGroupStart");
    TSA_SYM(groupEnd, "ncclGroupEnd");
    TSA_SYM(errStr, "ncclGetErrorString");
#undef TSA_SYM
    ok = N.getUniqueId && N.commInitRank && N.commDestroy && N.allGather && N.allReduce && N.broadcast && N.send &&
         N.recv && N.groupStart && N.groupEnd && N.errStr;
  });
  if (!ok) {
    cerr_set(err, errlen, "NCCL (libnccl.so.2) could not be loaded");
    return nullptr;
  }
  return &N;
}

}  // namespace

struct CommImpl {
  const Nccl* N = nullptr;
  ncclComm_t comm = nullptr;
  int device = 0;
  // device staging
  float* g_lc = nullptr;
  int* g_sc = nullptr;
  int* g_ns = nullptr;
  int ncap = 0;
  uint8_t* sendbuf = nullptr;
  uint8_t* recvbuf = nullptr;
  size_t send_cap = 0, recv_cap = 0;
  uint8_t* recbuf = nullptr;
  size_t rec_cap = 0;
  unsigned long long* u64buf = nullptr;
  double* dbuf = nullptr;
  size_t dcap = 0;
  int* d_idx = nullptr;
  int idx_cap = 0;
};

#define NCK(x)                                                                                  \
  do {                                                                                          \
    ncclResult_t r_ = (x);                                                                      \
    if (r_ != ncclSuccess) {                                                                    \
      cerr_set(err, errlen, "NCCL error %s at %s:%d", p->N->errStr(r_), __FILE__, __LINE__);   \
      return TSA_ERR_COMM;                                                                      \
    }                                                                                           \
  } while (0)
#define CCK(x)                                                                                  \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) {                                                                    \
      cerr_set(err, errlen, "CUDA error %s at %s:%d", cudaGetErrorString(e_), __FILE__, __LINE__); \
      return TSA_ERR_CUDA;                                                                      \
    }                                                                                           \
  } while (0)

template <typename T>
static int grow(T** buf, size_t* cap, size_t need, char* err, size_t errlen) {
  if (need <= *cap) return TSA_OK;
  cudaFree(*buf);
  *buf = nullptr;
  size_t n = std::max(need, *cap * 2);
  CCK(cudaMalloc(buf, n * sizeof(T)));
  *cap = n;
  return TSA_OK;
}

// Communicators are kept for the life of the process, keyed by (unique id, rank, world, device): a caller
// that passes the same id again (every rank does) reuses the communicator instead of re-initializing
// NCCL.  Two sessions must not use the same communicator at the same time.
namespace {
struct CommKey {
  char id[128];
  int rank, world, device;
  bool operator<(const CommKey& o) const {
    int c = memcmp(id, o.id, sizeof id);
    if (c) return c < 0;
    if (rank != o.rank) return rank < o.rank;
    if (world != o.world) return world < o.world;
    return device < o.device;
  }
};
std::mutex g_comm_mu;
std::map<CommKey, CommImpl*>& comm_cache() {
  static std::map<CommKey, CommImpl*> m;
  return m;
}
}  // namespace

Comm::~Comm() {}  // the cached CommImpl outlives the session

int comm_unique_id(void* id128, char* err, size_t errlen) {
  const Nccl* N = nccl(err, errlen);
  if (!N) return TSA_ERR_COMM;
  ncclUniqueId id;
  ncclResult_t r = N->getUniqueId(&id);
  if (r != ncclSuccess) {
    cerr_set(err, errlen, "ncclGetUniqueId: %s", N->errStr(r));
    return TSA_ERR_COMM;
  }
  memcpy(id128, &id, sizeof id);
  return TSA_OK;
}

int comm_create(const void* id128, int rank, int world, int device, Comm** out, char* err, size_t errlen) {
  *out = nullptr;
  if (!id128) {
    cerr_set(err, errlen, "world_size > 1 needs nccl_id");
    return TSA_ERR_ARG;
  }
  const Nccl* N = nccl(err, errlen);
  if (!N) return TSA_ERR_COMM;
  if (cudaSetDevice(device) != cudaSuccess) {
    cerr_set(err, errlen, "cudaSetDevice(%d) failed", device);
    return TSA_ERR_CUDA;
  }
  CommKey key;
  memcpy(key.id, id128, sizeof key.id);
  key.rank = rank;
  key.world = world;
  key.device = device;
  CommImpl* p = nullptr;
  {
    std::lock_guard<std::mutex> g(g_comm_mu);
    auto it = comm_cache().find(key);
    if (it != comm_cache().end()) p = it->second;
  }
  if (!p) {
    p = new CommImpl();
    p->N = N;
    p->device = device;
    ncclUniqueId id;
    memcpy(&id, id128, sizeof id);
    ncclResult_t r = N->commInitRank(&p->comm, world, id, rank);
    if (r != ncclSuccess) {
      cerr_set(err, errlen, "ncclCommInitRank: %s", N->errStr(r));
      delete p;
      return TSA_ERR_COMM;
    }
    std::lock_guard<std::mutex> g(g_comm_mu);
    comm_cache()[key] = p;
  }
  Comm* c = new Comm();
  c->p = p;
  c->rank = rank;
  c->world = world;
  *out = c;
  return TSA_OK;
}

int Comm::allgather_energies(const float* d_lc, const int* d_sc, const int* d_ns, int nloc, float* glc, int* gsc,
                             int* gns, cudaStream_t st, char* err, size_t errlen) {
  const int ng = nloc * world;
  if (p->ncap < ng) {
    cudaFree(p->g_lc);
    cudaFree(p->g_sc);
    cudaFree(p->g_ns);
    CCK(cudaMalloc(&p->g_lc, ng * sizeof(float)));
    CCK(cudaMalloc(&p->g_sc, ng * sizeof(int)));
    CCK(cudaMalloc(&p->g_ns, ng * sizeof(int)));
    p->ncap = ng;
  }
  NCK(p->N->groupStart());
  NCK(p->N->allGather(d_lc, p->g_lc, nloc, ncclFloat32, p->comm, st));
  NCK(p->N->allGather(d_sc, p->g_sc, nloc, ncclInt32, p->comm, st));
  NCK(p->N->allGather(d_ns, p->g_ns, nloc, ncclInt32, p->comm, st));
  NCK(p->N->groupEnd());
  CCK(cudaMemcpyAsync(glc, p->g_lc, ng * sizeof(float), cudaMemcpyDeviceToHost, st));
  CCK(cudaMemcpyAsync(gsc, p->g_sc, ng * sizeof(int), cudaMemcpyDeviceToHost, st));
  CCK(cudaMemcpyAsync(gns, p->g_ns, ng * sizeof(int), cudaMemcpyDeviceToHost, st));
  return TSA_OK;
}

int Comm::fetch_record(const uint8_t* d_rec_local, uint32_t bytes, int owner, uint8_t* host_out, cudaStream_t st,
                       char* err, size_t errlen) {
  int rc = grow(&p->recbuf, &p->rec_cap, bytes, err, errlen);
  if (rc) return rc;
  NCK(p->N->broadcast(rank == owner ? (const void*)d_rec_local : (const void*)p->recbuf, p->recbuf, bytes, ncclUint8,
                      owner, p->comm, st));
  CCK(cudaMemcpyAsync(host_out, p->recbuf, bytes, cudaMemcpyDeviceToHost, st));
  return TSA_OK;
}

int Comm::sum_u64(uint64_t* host_vals, int n, cudaStream_t st, char* err, size_t errlen) {
  size_t cap = p->u64buf ? 16 : 0;
  if (n > 16) {
    cerr_set(err, errlen, "sum_u64: at most 16 values");
    return TSA_ERR_ARG;
  }
  int rc = grow(&p->u64buf, &cap, 16, err, errlen);
  if (rc) return rc;
  CCK(cudaMemcpyAsync(p->u64buf, host_vals, n * 8, cudaMemcpyHostToDevice, st));
  NCK(p->N->allReduce(p->u64buf, p->u64buf, n, ncclUint64, ncclSum, p->comm, st));
  CCK(cudaMemcpyAsync(host_vals, p->u64buf, n * 8, cudaMemcpyDeviceToHost, st));
  CCK(cudaStreamSynchronize(st));
  return TSA_OK;
}

int Comm::allgather_host(const double* host_in, int n, double* host_out, cudaStream_t st, char* err,
                         size_t errlen) {
  const size_t tot = (size_t)n * (world + 1);  // [own n | gathered world*n]
  int rc = grow(&p->dbuf, &p->dcap, std::max<size_t>(tot, 1), err, errlen);
  if (rc) return rc;
  CCK(cudaMemcpyAsync(p->dbuf, host_in, (size_t)n * sizeof(double), cudaMemcpyHostToDevice, st));
  NCK(p->N->allGather(p->dbuf, p->dbuf + n, n, ncclFloat64, p->comm, st));
  CCK(cudaMemcpyAsync(host_out, p->dbuf + n, (size_t)n * world * sizeof(double), cudaMemcpyDeviceToHost, st));
  CCK(cudaStreamSynchronize(st));
  return TSA_OK;
}

int Comm::bcast_host(uint8_t* host, uint32_t bytes, int owner, cudaStream_t st, char* err, size_t errlen) {
  int rc = grow(&p->recbuf, &p->rec_cap, bytes, err, errlen);
  if (rc) return rc;
  if (rank == owner) CCK(cudaMemcpyAsync(p->recbuf, host, bytes, cudaMemcpyHostToDevice, st));
  NCK(p->N->broadcast(p->recbuf, p->recbuf, bytes, ncclUint8, owner, p->comm, st));
  if (rank != owner) CCK(cudaMemcpyAsync(host, p->recbuf, bytes, cudaMemcpyDeviceToHost, st));
  CCK(cudaStreamSynchronize(st));
  return TSA_OK;
}

int Comm::resample(const int* anc, uint8_t* d_rec, uint8_t* d_rec2, int* d_anc, int nloc, uint32_t rb,
                   cudaStream_t st, char* err, size_t errlen) {
  std::vector<int> src_of(nloc), send_off(world + 1), send_idx((size_t)nloc * world), recv_off(world + 1),
      recv_ids(nloc);
  tsa_resample_plan(anc, nloc, rank, world, src_of.data(), send_off.data(), send_idx.data(), recv_off.data(),
                    recv_ids.data());
  const int nsend = send_off[world], nrecv = recv_off[world];
  sent_bytes += (uint64_t)nsend * rb;
  recv_bytes += (uint64_t)nrecv * rb;
  int rc = grow(&p->sendbuf, &p->send_cap, (size_t)std::max(1, nsend) * rb, err, errlen);
  if (!rc) rc = grow(&p->recvbuf, &p->recv_cap, (size_t)std::max(1, nrecv) * rb, err, errlen);
  size_t icap = (size_t)p->idx_cap;
  if (!rc) rc = grow(&p->d_idx, &icap, (size_t)std::max(1, nsend), err, errlen);
  if (rc) return rc;
  p->idx_cap = (int)icap;
  // pack the records other ranks need, exchange them, then gather the new local population from
  // [local records ++ received records] (two sources, one gather kernel)
  if (nsend > 0) {
    CCK(cudaMemcpyAsync(p->d_idx, send_idx.data(), nsend * sizeof(int), cudaMemcpyHostToDevice, st));
    CCK(launch_copy_chains(d_rec, p->sendbuf, p->d_idx, nsend, rb, st));
  }
  uint8_t* recv_base = p->recvbuf;
  NCK(p->N->groupStart());
  for (int q = 0; q < world; q++) {
    if (q == rank) continue;
    int ns = send_off[q + 1] - send_off[q], nr = recv_off[q + 1] - recv_off[q];
    if (ns > 0) NCK(p->N->send(p->sendbuf + (size_t)send_off[q] * rb, (size_t)ns * rb, ncclUint8, q, p->comm, st));
    if (nr > 0) NCK(p->N->recv(recv_base + (size_t)recv_off[q] * rb, (size_t)nr * rb, ncclUint8, q, p->comm, st));
  }
  NCK(p->N->groupEnd());
  CCK(cudaMemcpyAsync(d_anc, src_of.data(), nloc * sizeof(int), cudaMemcpyHostToDevice, st));
  CCK(launch_copy_chains2(d_rec, nloc, recv_base, d_rec2, d_anc, nloc, rb, st));
  CCK(cudaStreamSynchronize(st));
  return TSA_OK;
}

}  // namespace tsa

extern "C" int tsa_resample_plan(const int* anc, int nloc, int rank, int world, int* src_of, int* send_off,
                                 int* send_idx, int* recv_off, int* recv_ids) {
  const int ng = nloc * world;
  // what this rank receives: distinct remote ancestors of its chains, grouped by owner
  std::vector<std::vector<int>> need(world), give(world);
  for (int c = 0; c < nloc; c++) {
    int a = anc[rank * nloc + c], q = a / nloc;
    if (q != rank) need[q].push_back(a);
  }
  // what this rank sends: for every other rank q, the distinct local ancestors of q's chains
  for (int q = 0; q < world; q++) {
    if (q == rank) continue;
    for (int c = 0; c < nloc; c++) {
      int a = anc[q * nloc + c];
      if (a / nloc == rank) give[q].push_back(a - rank * nloc);
    }
  }
  (void)ng;
  int k = 0;
  send_off[0] = 0;
  for (int q = 0; q < world; q++) {
    std::sort(give[q].begin(), give[q].end());
    give[q].erase(std::unique(give[q].begin(), give[q].end()), give[q].end());
    for (int x : give[q]) send_idx[k++] = x;
    send_off[q + 1] = k;
  }
  k = 0;
  recv_off[0] = 0;
  for (int q = 0; q < world; q++) {
    std::sort(need[q].begin(), need[q].end());
    need[q].erase(std::unique(need[q].begin(), need[q].end()), need[q].end());
    for (int x : need[q]) recv_ids[k++] = x;
    recv_off[q + 1] = k;
  }
  for (int c = 0; c < nloc; c++) {
    int a = anc[rank * nloc + c], q = a / nloc;
    if (q == rank) {
      src_of[c] = a - rank * nloc;
    } else {
      int pos = (int)(std::lower_bound(recv_ids + recv_off[q], recv_ids + recv_off[q + 1], a) - recv_ids);
      src_of[c] = nloc + pos;
    }
  }
  return 0;
}
