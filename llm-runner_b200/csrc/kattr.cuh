// Per-device, thread-safe one-time set-up of kernel attributes.
//
// CUDA keeps a kernel's cudaFuncAttributeMaxDynamicSharedMemorySize per
// device context: a process that drives several GPUs (one host thread per
// GPU, or one thread switching devices) must raise it on every device it
// launches on. `once_per_device(key, fn)` runs `fn` at most once per
// (key, current device) and remembers success; all host threads share the
// registry under one mutex, so two threads making their first call at the
// same time do not race. A failed `fn` is not remembered (the next call
// retries and reports the error again).
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <set>
#include <utility>

namespace llmr {

struct KernelAttrRegistry {
  std::mutex mu;
  std::set<std::pair<const void *, int>> done;
  std::map<const void *, int> regs;  // registers per thread at launch
};

inline KernelAttrRegistry &kernel_attr_registry() {
  static KernelAttrRegistry r;  // one instance for every translation unit
  return r;
}

// Runs fn() (returning cudaError_t) once per (key, current device).
template <typename Fn>
inline cudaError_t once_per_device(const void *key, Fn &&fn) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  KernelAttrRegistry &r = kernel_attr_registry();
  std::lock_guard<std::mutex> lock(r.mu);
  if (r.done.count({key, dev})) return cudaSuccess;
  e = fn();
  if (e == cudaSuccess) r.done.insert({key, dev});
  return e;
}

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per device.
template <typename Kernel>
inline cudaError_t set_smem_once(Kernel *kernel, int bytes) {
  const void *key = reinterpret_cast<const void *>(kernel);
  return once_per_device(key, [&]() {
    return cudaFuncSetAttribute(key, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
}

// Registers per thread that `kernel` is launched with (a property of the
// compiled code, the same on every sm_100 device), looked up once.
template <typename Kernel>
inline cudaError_t launch_regs(Kernel *kernel, int *out) {
  const void *key = reinterpret_cast<const void *>(kernel);
  KernelAttrRegistry &r = kernel_attr_registry();
  std::lock_guard<std::mutex> lock(r.mu);
  auto it = r.regs.find(key);
  if (it == r.regs.end()) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, key);
    if (e != cudaSuccess) return e;
    it = r.regs.emplace(key, fa.numRegs).first;
  }
  *out = it->second;
  return cudaSuccess;
}

}  // namespace llmr
