// Host-side helpers shared by the library's translation units: error
// propagation across the C ABI, memory-space detection, launch counting.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <utility>
#include <stdexcept>
#include <string>
#include <utility>

#include "../../include/se_gpu.h"

namespace se_gpu {

// Exception carrying one of the SE_ERR_* codes.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string &msg) : std::runtime_error(msg), code(c) {}
};

void set_last_error(const std::string &msg);
void clear_last_error();
void count_launch();

inline void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    const int code = e == cudaErrorMemoryAllocation ? SE_ERR_OUT_OF_MEMORY : SE_ERR_CUDA;
    throw Error(code, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// After a kernel launch: count it and surface launch-configuration errors.
inline void launched(const char *name) {
  count_launch();
  cuda_check(cudaGetLastError(), name);
}

// True when p is device (or managed) memory; false for pageable or pinned host memory.
inline bool is_device_ptr(const void *p) {
  if (p == nullptr) return false;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Makes `device` current for the scope and restores the previous device.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    cuda_check(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != device) cuda_check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

// Runs f, converting exceptions into a status code and a thread-local message.
template <class F> int guarded(F &&f) {
  try {
    clear_last_error();
    f();
    return SE_OK;
  } catch (const Error &e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::invalid_argument &e) {
    set_last_error(e.what());
    return SE_ERR_INVALID_ARGUMENT;
  } catch (const std::overflow_error &e) {
    set_last_error(e.what());
    return SE_ERR_OVERFLOW;
  } catch (const std::bad_alloc &) {
    set_last_error("host allocation failed");
    return SE_ERR_OUT_OF_MEMORY;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return SE_ERR_RUNTIME;
  }
}

inline size_t key_bytes(int key_dtype) { return key_dtype <= SE_KEY_UINT32 ? 4 : 8; }
inline size_t value_bytes(int value_dtype) { return value_dtype == SE_FLOAT32 ? 4 : 2; }

// Launches a kernel that may start while the previous kernel on the stream
// finishes (programmatic dependent launch): its blocks are scheduled as the
// previous grid's blocks retire and wait in pdl_wait() (griddepcontrol.wait)
// for that grid's completion and memory, so the launch latency of a chain of
// short kernels overlaps their tails. Captured into graphs as programmatic
// edges. Every kernel launched this way calls pdl_wait() before it touches
// memory the previous kernels write or read.
template <class... KArgs, class... Args>
inline void pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cuda_check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), "cudaLaunchKernelEx");
}

// Lets `kernel` take up to `bytes` of dynamic shared memory (beyond the
// default 48 KB of static plus dynamic). The attribute only grows: it is
// set when a launch needs more than any before on this device (the first
// such call; a graph capture of the same sizes then finds it set).
template <class... KArgs>
inline void allow_dynamic_smem(void (*kernel)(KArgs...), size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void *, int>, size_t> allowed;
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  const auto key = std::make_pair(reinterpret_cast<const void *>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = allowed.find(key);
  if (it != allowed.end() && it->second >= bytes) return;
  cuda_check(cudaFuncSetAttribute(reinterpret_cast<const void *>(kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(bytes)),
             "cudaFuncSetAttribute");
  allowed[key] = bytes;
}

inline unsigned grid_for(size_t work_items, unsigned per_block, unsigned cap = 1u << 20) {
  size_t b = (work_items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > cap) b = cap;
  return unsigned(b);
}

}  // namespace se_gpu
