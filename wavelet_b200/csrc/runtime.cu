// Per-device error word that every kernel of the extension reports into, and
// small runtime queries used by the Python layer.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <stdexcept>

#include "common.cuh"

namespace wb {

int* error_word(int device) {
  static int* words[64] = {nullptr};
  static std::mutex mu;
  if (device < 0 || device >= 64) throw std::runtime_error("wavelet_b200: bad device index");
  if (words[device]) return words[device];
  std::lock_guard<std::mutex> lock(mu);
  if (!words[device]) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess)
      throw std::runtime_error("wavelet_b200: cannot allocate the device error word");
    cudaMemset(p, 0, sizeof(int));
    cudaDeviceSynchronize();
    words[device] = p;
    cudaSetDevice(prev);
  }
  return words[device];
}

static std::atomic<long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

void note_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int read_error_word(int device) {
  int v = 0;
  cudaMemcpy(&v, error_word(device), sizeof(int), cudaMemcpyDeviceToHost);
  return v;
}

void clear_error_word(int device) { cudaMemset(error_word(device), 0, sizeof(int)); }

}  // namespace wb
