// tsa_spectral.cu -- the spectral start trees' two numerical parts on the GPU (the ordering search itself
// stays in treesa_gpu_b200/spectral.py, as the reference's treesa_gpu/spectral.py does it in Python):
//
//   tsa_laplacian_vectors: the low eigenvectors of the tensor graph's Laplacian (the reference's
//     laplacian_vectors: dense numpy.linalg.eigh / scipy eigsh).  The dense Laplacian is built on the
//     device and cuSOLVER's syevdx computes only eigenpairs 2..k+1.  cuSOLVER is loaded with dlopen (the
//     copy the process already holds, else the toolkit's), so the library has no link-time dependency.
//   tsa_path_costs: the exact (tc, sc) of the path tree of each of a batch of tensor orderings (the
//     reference's path_cost), one CTA per ordering.
#include <cuda_runtime.h>
#include <cusolverDn.h>
#include <dlfcn.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "../../include/treesa_b200.h"

namespace {

void fail(char* err, size_t n, const char* fmt, ...) {
  if (!err || !n) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, n, fmt, ap);
  va_end(ap);
}

struct Cusolver {
  decltype(&cusolverDnCreate) create = nullptr;
  decltype(&cusolverDnDestroy) destroy = nullptr;
  decltype(&cusolverDnSetStream) set_stream = nullptr;
  decltype(&cusolverDnDsyevdx_bufferSize) evdx_buffer = nullptr;
  decltype(&cusolverDnDsyevdx) evdx = nullptr;
  bool ok = false;
};

const Cusolver& cusolver() {
  static Cusolver C;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libcusolver.so.11", "/usr/local/cuda/lib64/libcusolver.so.11", "libcusolver.so"};
    void* h = nullptr;
    for (const char* n : names)
      if ((h = dlopen(n, RTLD_NOW | RTLD_LOCAL))) break;
    if (!h) return;
    C.create = reinterpret_cast<decltype(C.create)>(dlsym(h, "cusolverDnCreate"));
    C.destroy = reinterpret_cast<decltype(C.destroy)>(dlsym(h, "cusolverDnDestroy"));
    C.set_stream = reinterpret_cast<decltype(C.set_stream)>(dlsym(h, "cusolverDnSetStream"));
    C.evdx_buffer = reinterpret_cast<decltype(C.evdx_buffer)>(dlsym(h, "cusolverDnDsyevdx_bufferSize"));
    C.evdx = reinterpret_cast<decltype(C.evdx)>(dlsym(h, "cusolverDnDsyevdx"));
    C.ok = C.create && C.destroy && C.set_stream && C.evdx_buffer && C.evdx;
  });
  return C;
}

// Per-device workspace kept for the process (the ordering search calls tsa_path_costs dozens of times in a
// row): a stream, grow-only device buffers, pinned staging for the orderings and results, and the cuSOLVER
// handle.  Calls on one device are serialised by its mutex.
struct Workspace {
  std::mutex mu;
  cudaStream_t st = nullptr;
  cusolverDnHandle_t solver = nullptr;
  void* dbuf[8] = {};
  size_t dcap[8] = {};
  void* hbuf[2] = {};
  size_t hcap[2] = {};
};
constexpr int kMaxDevices = 64;
Workspace g_ws[kMaxDevices];

// device buffer slot i of at least n bytes (contents not kept)
cudaError_t dgrow(Workspace& W, int i, size_t n, void** p) {
  if (W.dcap[i] < n) {
    if (W.dbuf[i]) cudaFree(W.dbuf[i]);
    W.dbuf[i] = nullptr;
    W.dcap[i] = 0;
    const size_t cap = n + n / 2 + 256;
    cudaError_t e = cudaMalloc(&W.dbuf[i], cap);
    if (e != cudaSuccess) return e;
    W.dcap[i] = cap;
  }
  *p = W.dbuf[i];
  return cudaSuccess;
}
cudaError_t hgrow(Workspace& W, int i, size_t n, void** p) {
  if (W.hcap[i] < n) {
    if (W.hbuf[i]) cudaFreeHost(W.hbuf[i]);
    W.hbuf[i] = nullptr;
    W.hcap[i] = 0;
    const size_t cap = n + n / 2 + 256;
    cudaError_t e = cudaMallocHost(&W.hbuf[i], cap);
    if (e != cudaSuccess) return e;
    W.hcap[i] = cap;
  }
  *p = W.hbuf[i];
  return cudaSuccess;
}

// L = D - W for the pair list (r, c, w) (each unordered pair once), L row-major n x n (symmetric)
__global__ void k_laplacian_offdiag(double* L, double* deg, int n, int nnz, const int32_t* r, const int32_t* c,
                                    const double* w) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nnz; e += gridDim.x * blockDim.x) {
    const int a = r[e], b = c[e];
    const double x = w[e];
    atomicAdd(&L[(size_t)a * n + b], -x);
    atomicAdd(&L[(size_t)b * n + a], -x);
    atomicAdd(&deg[a], x);
    atomicAdd(&deg[b], x);
  }
}
__global__ void k_laplacian_diag(double* L, const double* deg, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    L[(size_t)i * n + i] += deg[i];
}

// One ordering per CTA.  Tensor order[i] is contracted at step i into the prefix.  With first[l] / last[l]
// the positions of label l's first and last tensor (open labels: last = m), the labels alive across the
// cut before position c are those with first < c <= last; step i (i >= 2) costs alive[i] + new[i] (new:
// labels first seen at i), step 1 the union of the first two tensors; the output of step i is alive[i+1].
// tc = log2 sum 2^cost, sc = max(outputs, input tensor sizes).  Scratch: pos[m], first/last[L], diff[m+2],
// newc[m] per ordering (global).
__global__ void __launch_bounds__(256) k_path_costs(int m, int nlab, const int32_t* ix_off, const int32_t* ix_lab,
                                                    const uint8_t* open, const int32_t* orders, int32_t* scratch,
                                                    int max_tensor, double* tc_out, int32_t* sc_out) {
  const int b = blockIdx.x, tid = threadIdx.x, T = blockDim.x;
  const int32_t* ord = orders + (size_t)b * m;
  int32_t* pos = scratch + (size_t)b * (3 * (size_t)m + 2 + 2 * (size_t)nlab);
  int32_t* first = pos + m;
  int32_t* last = first + nlab;
  int32_t* diff = last + nlab;  // m + 2
  int32_t* newc = diff + m + 2;
  for (int i = tid; i < m; i += T) {
    pos[ord[i]] = i;
    newc[i] = 0;
  }
  for (int i = tid; i < m + 2; i += T) diff[i] = 0;
  for (int l = tid; l < nlab; l += T) {
    first[l] = m;
    last[l] = -1;
  }
  __syncthreads();
  for (int t = tid; t < m; t += T) {
    const int p = pos[t];
    for (int q = ix_off[t]; q < ix_off[t + 1]; q++) {
      atomicMin(&first[ix_lab[q]], p);
      atomicMax(&last[ix_lab[q]], p);
    }
  }
  __syncthreads();
  for (int l = tid; l < nlab; l += T) {
    const int f = first[l];
    if (f >= m) continue;  // in no tensor
    const int la = open[l] ? m : last[l];
    atomicAdd(&diff[f + 1], 1);
    atomicAdd(&diff[la + 1], -1);
    atomicAdd(&newc[f], 1);
  }
  __syncthreads();
  // alive[c] = diff[0] + ... + diff[c] (c = 0..m), written over diff by one thread: independent loads and
  // stores around a running sum in a register (the scan is not where the time goes)
  if (tid == 0) {
    int acc = 0;
    for (int c = 0; c <= m; c++) {
      acc += diff[c];
      diff[c] = acc;
    }
  }
  __syncthreads();
  const int32_t* alive = diff;
  // costs of steps 1..m-1: maximum first, then the sum of 2^(cost - max)
  __shared__ int s_red[256];
  __shared__ double s_sum[256];
  auto cost_of = [&](int i) { return i == 1 ? newc[0] + newc[1] : alive[i] + newc[i]; };
  int cm = 0, so = 0;
  for (int i = 1 + tid; i < m; i += T) cm = max(cm, cost_of(i));
  for (int i = 2 + tid; i <= m; i += T) so = max(so, alive[i]);
  s_red[tid] = cm;
  __syncthreads();
  for (int o = T / 2; o > 0; o >>= 1) {
    if (tid < o) s_red[tid] = max(s_red[tid], s_red[tid + o]);
    __syncthreads();
  }
  cm = s_red[0];
  __syncthreads();
  s_red[tid] = so;
  double sum = 0;
  for (int i = 1 + tid; i < m; i += T) sum += exp2((double)(cost_of(i) - cm));
  s_sum[tid] = sum;
  __syncthreads();
  for (int o = T / 2; o > 0; o >>= 1) {
    if (tid < o) {
      s_red[tid] = max(s_red[tid], s_red[tid + o]);
      s_sum[tid] += s_sum[tid + o];
    }
    __syncthreads();
  }
  if (tid == 0) {
    tc_out[b] = (double)cm + log2(s_sum[0]);
    sc_out[b] = max(s_red[0], max_tensor);
  }
}

}  // namespace

extern "C" int tsa_laplacian_vectors(int32_t n, int32_t nnz, const int32_t* rows, const int32_t* cols,
                                     const double* w, int32_t k, int32_t device, double* V, char* err,
                                     size_t errlen) {
  if (n < 3 || nnz < 0 || k < 1 || k > n - 2 || !V || (nnz > 0 && (!rows || !cols || !w))) {
    fail(err, errlen, "tsa_laplacian_vectors: need n >= 3, 1 <= k <= n - 2 and the pair list");
    return TSA_ERR_ARG;
  }
  if ((size_t)n * (size_t)n * 8 > (size_t)32 << 30) {
    fail(err, errlen, "tsa_laplacian_vectors: %d tensors exceed the dense eigensolver's 32 GiB", n);
    return TSA_ERR_UNSUPPORTED;
  }
  const Cusolver& S = cusolver();
  if (!S.ok) {
    fail(err, errlen, "tsa_laplacian_vectors: cuSOLVER (libcusolver.so.11) could not be loaded");
    return TSA_ERR_UNSUPPORTED;
  }
  if (device < 0 || device >= kMaxDevices) {
    fail(err, errlen, "tsa_laplacian_vectors: device %d out of range", device);
    return TSA_ERR_ARG;
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    fail(err, errlen, "tsa_laplacian_vectors: cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    return TSA_ERR_CUDA;
  }
  Workspace& Wk = g_ws[device];
  std::lock_guard<std::mutex> lock(Wk.mu);
  cudaStream_t st = Wk.st;
  cusolverDnHandle_t h = Wk.solver;
  double *dL = nullptr, *ddeg = nullptr, *dW = nullptr, *dwork = nullptr, *dw = nullptr;
  int32_t *dr = nullptr, *dc = nullptr;
  int* dinfo = nullptr;
  int rc = TSA_OK;
  int meig = 0, lwork = 0, info = 0;
  auto ck = [&](cudaError_t x, const char* what) {
    if (x != cudaSuccess && rc == TSA_OK) {
      fail(err, errlen, "tsa_laplacian_vectors: %s: %s", what, cudaGetErrorString(x));
      rc = TSA_ERR_CUDA;
    }
    return rc == TSA_OK;
  };
  auto cs = [&](cusolverStatus_t x, const char* what) {
    if (x != CUSOLVER_STATUS_SUCCESS && rc == TSA_OK) {
      fail(err, errlen, "tsa_laplacian_vectors: %s failed (cuSOLVER status %d)", what, (int)x);
      rc = TSA_ERR_CUDA;
    }
    return rc == TSA_OK;
  };
  const size_t nn = (size_t)n * n;
  if ((st || ck(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream")) && (Wk.st = st) &&
      ck(cudaMalloc(&dL, nn * 8), "cudaMalloc") && ck(cudaMalloc(&ddeg, (size_t)n * 8), "cudaMalloc") &&
      ck(cudaMalloc(&dW, (size_t)n * 8), "cudaMalloc") && ck(cudaMalloc(&dinfo, sizeof(int)), "cudaMalloc") &&
      ck(cudaMalloc(&dr, sizeof(int32_t) * (nnz + 1)), "cudaMalloc") &&
      ck(cudaMalloc(&dc, sizeof(int32_t) * (nnz + 1)), "cudaMalloc") &&
      ck(cudaMalloc(&dw, sizeof(double) * (nnz + 1)), "cudaMalloc") &&
      ck(cudaMemsetAsync(dL, 0, nn * 8, st), "memset") && ck(cudaMemsetAsync(ddeg, 0, (size_t)n * 8, st), "memset")) {
    if (nnz > 0) {
      ck(cudaMemcpyAsync(dr, rows, sizeof(int32_t) * nnz, cudaMemcpyHostToDevice, st), "copy");
      ck(cudaMemcpyAsync(dc, cols, sizeof(int32_t) * nnz, cudaMemcpyHostToDevice, st), "copy");
      ck(cudaMemcpyAsync(dw, w, sizeof(double) * nnz, cudaMemcpyHostToDevice, st), "copy");
      k_laplacian_offdiag<<<(nnz + 255) / 256 < 4096 ? (nnz + 255) / 256 : 4096, 256, 0, st>>>(dL, ddeg, n, nnz, dr,
                                                                                               dc, dw);
      ck(cudaGetLastError(), "laplacian");
    }
    k_laplacian_diag<<<(n + 255) / 256, 256, 0, st>>>(dL, ddeg, n);
    ck(cudaGetLastError(), "laplacian");
    if (rc == TSA_OK && (h || cs(S.create(&h), "cusolverDnCreate")) && (Wk.solver = h) &&
        cs(S.set_stream(h, st), "cusolverDnSetStream") &&
        cs(S.evdx_buffer(h, CUSOLVER_EIG_MODE_VECTOR, CUSOLVER_EIG_RANGE_I, CUBLAS_FILL_MODE_LOWER, n, dL, n, 0.0,
                         0.0, 2, k + 1, &meig, dW, &lwork),
           "syevdx_bufferSize") &&
        ck(cudaMalloc(&dwork, sizeof(double) * (size_t)(lwork > 0 ? lwork : 1)), "cudaMalloc") &&
        cs(S.evdx(h, CUSOLVER_EIG_MODE_VECTOR, CUSOLVER_EIG_RANGE_I, CUBLAS_FILL_MODE_LOWER, n, dL, n, 0.0, 0.0, 2,
                  k + 1, &meig, dW, dwork, lwork, dinfo),
           "syevdx") &&
        ck(cudaMemcpyAsync(&info, dinfo, sizeof(int), cudaMemcpyDeviceToHost, st), "copy") &&
        ck(cudaStreamSynchronize(st), "sync")) {
      if (info != 0 || meig != k) {
        fail(err, errlen, "tsa_laplacian_vectors: syevdx info %d, %d of %d eigenpairs", info, meig, k);
        rc = TSA_ERR_CUDA;
      } else {
        // column j of A (column-major) is eigenvector 2 + j; V is row-major [n][k]
        std::vector<double> col((size_t)n * k);
        if (ck(cudaMemcpy(col.data(), dL, sizeof(double) * (size_t)n * k, cudaMemcpyDeviceToHost), "copy"))
          for (int j = 0; j < k; j++)
            for (int i = 0; i < n; i++) V[(size_t)i * k + j] = col[(size_t)j * n + i];
      }
    }
  }
  cudaFree(dL);
  cudaFree(ddeg);
  cudaFree(dW);
  cudaFree(dwork);
  cudaFree(dinfo);
  cudaFree(dr);
  cudaFree(dc);
  cudaFree(dw);
  return rc;
}

extern "C" int tsa_path_costs(const tsa_instance* inst, int32_t norders, const int32_t* orders, int32_t device,
                              double* tc, int32_t* sc, char* err, size_t errlen) {
  if (!inst || !orders || !tc || !sc || norders < 1 || inst->m < 2 || !inst->ix_offsets || inst->nlab < 0) {
    fail(err, errlen, "tsa_path_costs: need an instance with m >= 2 and at least one ordering");
    return TSA_ERR_ARG;
  }
  const int m = inst->m, nlab = inst->nlab > 0 ? inst->nlab : 1, nocc = inst->ix_offsets[m];
  std::vector<uint8_t> open(nlab, 0);
  for (int q = 0; q < inst->niy; q++)
    if (inst->iy[q] >= 0 && inst->iy[q] < nlab) open[inst->iy[q]] = 1;
  int max_tensor = 0;
  for (int t = 0; t < m; t++) max_tensor = std::max(max_tensor, inst->ix_offsets[t + 1] - inst->ix_offsets[t]);
  for (int t = 0; t < m; t++)
    for (int q = inst->ix_offsets[t]; q < inst->ix_offsets[t + 1]; q++)
      if (inst->ix_labels[q] < 0 || inst->ix_labels[q] >= nlab) {
        fail(err, errlen, "tsa_path_costs: label out of range");
        return TSA_ERR_ARG;
      }
  for (size_t i = 0; i < (size_t)norders * m; i++)
    if (orders[i] < 0 || orders[i] >= m) {
      fail(err, errlen, "tsa_path_costs: ordering entry out of range");
      return TSA_ERR_ARG;
    }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    fail(err, errlen, "tsa_path_costs: cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    return TSA_ERR_CUDA;
  }
  if (device < 0 || device >= kMaxDevices) {
    fail(err, errlen, "tsa_path_costs: device %d out of range", device);
    return TSA_ERR_ARG;
  }
  Workspace& W = g_ws[device];
  std::lock_guard<std::mutex> lock(W.mu);
  const size_t per = 3 * (size_t)m + 2 + 2 * (size_t)nlab;
  int32_t *doff = nullptr, *dlab = nullptr, *dord = nullptr, *dscr = nullptr, *dsc = nullptr;
  uint8_t* dopen = nullptr;
  double* dtc = nullptr;
  void* hord = nullptr;
  void* hout = nullptr;
  const size_t obytes = sizeof(int32_t) * (size_t)norders * m, rbytes = (sizeof(double) + 4) * (size_t)norders;
  if (!W.st) e = cudaStreamCreateWithFlags(&W.st, cudaStreamNonBlocking);
  cudaStream_t st = W.st;
  auto go = [&](cudaError_t x) {
    if (e == cudaSuccess) e = x;
    return e == cudaSuccess;
  };
  if (go(dgrow(W, 0, sizeof(int32_t) * (m + 1), (void**)&doff)) &&
      go(dgrow(W, 1, sizeof(int32_t) * (nocc + 1), (void**)&dlab)) && go(dgrow(W, 2, obytes, (void**)&dord)) &&
      go(dgrow(W, 3, sizeof(int32_t) * per * norders, (void**)&dscr)) &&
      go(dgrow(W, 4, sizeof(int32_t) * norders, (void**)&dsc)) && go(dgrow(W, 5, nlab, (void**)&dopen)) &&
      go(dgrow(W, 6, sizeof(double) * norders, (void**)&dtc)) && go(hgrow(W, 0, obytes, &hord)) &&
      go(hgrow(W, 1, rbytes, &hout))) {
    memcpy(hord, orders, obytes);
    double* htc = static_cast<double*>(hout);
    int32_t* hsc = reinterpret_cast<int32_t*>(htc + norders);
    if (go(cudaMemcpyAsync(doff, inst->ix_offsets, sizeof(int32_t) * (m + 1), cudaMemcpyHostToDevice, st)) &&
        (nocc == 0 ||
         go(cudaMemcpyAsync(dlab, inst->ix_labels, sizeof(int32_t) * nocc, cudaMemcpyHostToDevice, st))) &&
        go(cudaMemcpyAsync(dord, hord, obytes, cudaMemcpyHostToDevice, st)) &&
        go(cudaMemcpyAsync(dopen, open.data(), nlab, cudaMemcpyHostToDevice, st))) {
      k_path_costs<<<norders, 256, 0, st>>>(m, nlab, doff, dlab, dopen, dord, dscr, max_tensor, dtc, dsc);
      if (go(cudaGetLastError()) &&
          go(cudaMemcpyAsync(htc, dtc, sizeof(double) * norders, cudaMemcpyDeviceToHost, st)) &&
          go(cudaMemcpyAsync(hsc, dsc, sizeof(int32_t) * norders, cudaMemcpyDeviceToHost, st)) &&
          go(cudaStreamSynchronize(st))) {
        memcpy(tc, htc, sizeof(double) * norders);
        memcpy(sc, hsc, sizeof(int32_t) * norders);
      }
    }
  }
  if (e != cudaSuccess) {
    fail(err, errlen, "tsa_path_costs: CUDA error %s", cudaGetErrorString(e));
    return TSA_ERR_CUDA;
  }
  return TSA_OK;
}
