// Allocation-free attention backward (see attention_noalloc.h for who needs
// it and why).  This file has no counterpart in the reference project.
//
// The Delta scratch (Hq x T floats) and the kernels' error word are
// file-scope static device arrays.  In host code their names are only
// host-side stand-ins, never device addresses, so the device address of each
// is resolved once per device with cudaGetSymbolAddress (that device current)
// and cached; kernels only ever receive those resolved addresses.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "attention.h"
#include "attention_noalloc.h"

namespace {

static __device__ __align__(256) float g_noalloc_delta[WB_ATTN_BWD_NOALLOC_MAX_ROWS];
static __device__ __align__(256) int g_noalloc_err[1];

constexpr int kMaxDevices = 64;
// Resolved addresses per device.  Readers on any host thread load them with
// acquire; the one writer (under the mutex) publishes each with release after
// cudaGetSymbolAddress succeeded, so a non-null value is always complete.
std::atomic<float*> g_delta_addr[kMaxDevices];
std::atomic<int*> g_err_addr[kMaxDevices];
std::mutex g_setup_mu;

// Resolve the static arrays' device addresses for the current device.
int setup_current_device(int* dev_out, float** delta, int** err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return WB_NOALLOC_ESETUP;
  *dev_out = dev;
  float* d = g_delta_addr[dev].load(std::memory_order_acquire);
  int* e = g_err_addr[dev].load(std::memory_order_acquire);
  if (!d || !e) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    d = g_delta_addr[dev].load(std::memory_order_relaxed);
    if (!d) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_delta) != cudaSuccess || p == nullptr) return WB_NOALLOC_ESETUP;
      d = static_cast<float*>(p);
      g_delta_addr[dev].store(d, std::memory_order_release);
    }
    e = g_err_addr[dev].load(std::memory_order_relaxed);
    if (!e) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_err) != cudaSuccess || p == nullptr) return WB_NOALLOC_ESETUP;
      e = static_cast<int*>(p);
      g_err_addr[dev].store(e, std::memory_order_release);
    }
  }
  *delta = d;
  *err = e;
  return WB_NOALLOC_OK;
}

}  // namespace

extern "C" int wb_attn_bwd_noalloc(const void* q, int64_t q_row, const void* k, int64_t k_row, const void* v,
                                   int64_t v_row, const void* o, int64_t o_row, const float* lse, const void* dout,
                                   void* dq, void* dk, void* dv, const int* cu_seqlens, int nseq, int max_seqlen,
                                   int T, int Hq, int Hk, float scale, cudaStream_t stream) {
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv || !cu_seqlens) return WB_NOALLOC_EARG;
  if (T < 0 || nseq < 0 || Hq <= 0 || Hk <= 0 || Hq % Hk != 0 || max_seqlen < 0) return WB_NOALLOC_EARG;
  if ((int64_t)Hq * (int64_t)T > (int64_t)WB_ATTN_BWD_NOALLOC_MAX_ROWS) return WB_NOALLOC_ETOO_LARGE;
  int dev = 0;
  float* delta = nullptr;
  int* err = nullptr;
  const int rc = setup_current_device(&dev, &delta, &err);
  if (rc != WB_NOALLOC_OK) return rc;
  if (T == 0 || nseq == 0) return WB_NOALLOC_OK;
  // The error word must start at zero for this call; Delta is fully
  // overwritten by the pre-pass before it is read, so it needs no clearing.
  if (cudaMemsetAsync(err, 0, sizeof(int), stream) != cudaSuccess) return WB_NOALLOC_ELAUNCH;
  wb::AttnBwdArgs b;
  b.f.q = q;
  b.f.k = k;
  b.f.v = v;
  b.f.q_row = q_row;
  b.f.k_row = k_row;
  b.f.v_row = v_row;
  b.f.o = const_cast<void*>(o);
  b.f.o_row = o_row;
  b.f.lse = const_cast<float*>(lse);
  b.f.cu_seqlens = cu_seqlens;
  b.f.nseq = nseq;
  b.f.max_seqlen = max_seqlen;
  b.f.T = T;
  b.f.Hq = Hq;
  b.f.Hk = Hk;
  b.f.head_dim = 128;
  b.f.scale = scale;
  b.dout = dout;
  b.dq = dq;
  b.dk = dk;
  b.dv = dv;
  b.delta = delta;
  const int lrc = wb::attn_bwd_explicit(b, err, stream);
  if (lrc == 1) return WB_NOALLOC_EARG;
  return lrc == 0 ? WB_NOALLOC_OK : WB_NOALLOC_ELAUNCH;
}

extern "C" int wb_attn_bwd_noalloc_status(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  int* err = g_err_addr[device].load(std::memory_order_acquire);
  if (!err) return 0;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int v = 0;
  cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaSetDevice(prev);
  return v;
}

extern "C" const char* wb_attn_bwd_noalloc_strerror(int code) {
  switch (code) {
    case WB_NOALLOC_OK:
      return "ok";
    case WB_NOALLOC_ETOO_LARGE:
      return "Hq * T exceeds the static scratch capacity (WB_ATTN_BWD_NOALLOC_MAX_ROWS = 1048576 rows)";
    case WB_NOALLOC_EARG:
      return "invalid argument (a null pointer, negative T, nseq or max_seqlen, Hq or Hk not positive, or Hq "
             "not a multiple of Hk)";
    case WB_NOALLOC_ESETUP:
      return "could not resolve the device address of the static scratch (cudaGetSymbolAddress failed)";
    case WB_NOALLOC_ELAUNCH:
      return "kernel launch or TMA descriptor encoding failed";
    default:
      return "unknown error";
  }
}
