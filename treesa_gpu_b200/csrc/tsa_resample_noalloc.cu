// tsa_resample_noalloc.cu -- population resampling that allocates nothing.
//
// tsa_resample gathers every chain record's ancestor through a scratch copy of the population that it
// allocates with cudaMalloc for the call.  Some callers cannot allocate device memory at that point: a
// serving process whose device memory is owned by its own fixed pool after start-up, or a latency-bound
// loop where cudaMalloc/cudaFree would synchronize the device and stall the work queued around it.  tsa_resample_noalloc does the same gather
// through scratch space that the library reserves once, in this file: a static device array of
// kScratchBytes bytes of records and kMaxChains ancestor slots, held by every GPU that loads this code
// until the process exits.
//
// Set-up: the first call on a device (with that device current) looks the arrays up with
// cudaGetSymbolAddress and caches the addresses; make that first call before any stream capture.
// Every call shares the arrays and leaves the last call's data in them; nothing in them has to start at
// zero (a call reads only bytes it has written first), but two calls that overlap on the GPU (different
// streams, or a second call before the first has finished) race on the same scratch.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "../../include/treesa_b200.h"

namespace {

constexpr size_t kScratchBytes = size_t(64) << 20;  // 64 MiB of chain records
constexpr int kMaxChains = 65536;                   // ancestor slots

static __device__ __align__(256) uint8_t g_rec_scratch[kScratchBytes];
static __device__ __align__(256) int32_t g_anc_scratch[kMaxChains];

// dst chain c <- src chain anc[c] (the gather of k_copy, with both tables in the static scratch)
__global__ void k_gather_noalloc(const uint4* __restrict__ src, uint4* __restrict__ dst, const int32_t* __restrict__ anc,
                                 int n4) {
  const uint4* s = src + (size_t)anc[blockIdx.x] * n4;
  uint4* d = dst + (size_t)blockIdx.x * n4;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d[i] = s[i];
}

struct DeviceScratch {
  uint8_t* rec = nullptr;
  int32_t* anc = nullptr;
};
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];

void fail(char* err, size_t n, const char* fmt, ...) {
  if (!err || !n) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, n, fmt, ap);
  va_end(ap);
}

// The device addresses of the scratch arrays on the current device (looked up once per device).
int scratch_for_current_device(DeviceScratch* out, char* err, size_t errlen) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    fail(err, errlen, "tsa_resample_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return TSA_ERR_CUDA;
  }
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& d = g_dev[dev];
  if (!d.rec) {
    uint8_t* rec = nullptr;
    int32_t* anc = nullptr;
    e = cudaGetSymbolAddress((void**)&rec, g_rec_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&anc, g_anc_scratch);
    if (e != cudaSuccess) {
      fail(err, errlen, "tsa_resample_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
           cudaGetErrorString(e));
      return TSA_ERR_CUDA;
    }
    d.rec = rec;
    d.anc = anc;
  }
  *out = d;
  return TSA_OK;
}

}  // namespace

extern "C" int tsa_resample_noalloc(void* records, const int32_t* anc, int32_t nchains, uint32_t rec_bytes,
                                    void* stream, char* err, size_t errlen) {
  if (!records || !anc || nchains < 1 || rec_bytes == 0 || rec_bytes % 16) {
    fail(err, errlen, "tsa_resample_noalloc: need records, anc, nchains >= 1 and rec_bytes a positive multiple of 16");
    return TSA_ERR_ARG;
  }
  if (nchains > kMaxChains || (size_t)nchains * rec_bytes > kScratchBytes) {
    fail(err, errlen,
         "tsa_resample_noalloc: %d chains of %u bytes exceed the built-in scratch (at most %d chains and %zu bytes "
         "in all); use tsa_resample",
         nchains, rec_bytes, kMaxChains, kScratchBytes);
    return TSA_ERR_ARG;
  }
  for (int c = 0; c < nchains; c++)
    if (anc[c] < 0 || anc[c] >= nchains) {
      fail(err, errlen, "tsa_resample_noalloc: ancestor %d of chain %d out of range", anc[c], c);
      return TSA_ERR_ARG;
    }
  DeviceScratch sc;
  int rc = scratch_for_current_device(&sc, err, errlen);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t bytes = (size_t)nchains * rec_bytes;
  cudaError_t e = cudaMemcpyAsync(sc.anc, anc, (size_t)nchains * sizeof(int32_t), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    k_gather_noalloc<<<nchains, 256, 0, st>>>(static_cast<const uint4*>(records), reinterpret_cast<uint4*>(sc.rec),
                                               sc.anc, (int)(rec_bytes / 16));
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(records, sc.rec, bytes, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    fail(err, errlen, "tsa_resample_noalloc: CUDA error %s", cudaGetErrorString(e));
    return TSA_ERR_CUDA;
  }
  return TSA_OK;
}
