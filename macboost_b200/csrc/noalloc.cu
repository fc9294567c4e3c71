// macboost_predict_device_noalloc: predict from device memory without any
// device allocation (declared in include/macboost_c.h).
//
// Who needs it: hosts that own every byte of GPU memory through their own pool
// (serving stacks that reserve most of HBM up front, so a library cudaMalloc
// fails or fragments their pool), and latency-sensitive pipelines in which a
// library's cudaMalloc / cudaFree -- which can synchronise the whole device --
// would stall other streams.  They prepare the model once (macboost_prepare,
// which does allocate, at load time) and afterwards score through this entry
// point, which allocates nothing.
//
// The scratch it needs lives in one file-scope __device__ array below: a
// status word the kernel reports waiting failures into, the kernel's two
// row-chunk counters (which every launch leaves at zero), and room for the
// feature-major copy of row-major input (at most kRowMajorBytes).  Every GPU
// that loads this module keeps the array until the process exits.  All calls
// share it and it keeps the previous call's contents, so each call clears the
// status word first, and calls that overlap on the GPU (other streams, other
// host threads) race on it: serialise them.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/macboost_c.h"
#include "engine.h"
#include "kernels.h"

namespace {

constexpr size_t kStatusBytes = 256;                   // status word, padded
constexpr size_t kRowMajorBytes = size_t(16) << 20;    // 16 MiB = 4,194,304 floats
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kStatusBytes + kRowMajorBytes];

std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};  // device address of the scratch, per device

// Device address of the scratch on the current device (= `device`), looked up
// once per device.  In host code the array's name is only a stand-in for it.
int scratch_address(int device, void** out, std::string& err) {
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (g_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t ce = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (ce != cudaSuccess || p == nullptr) {
      err = std::string("cudaGetSymbolAddress (no-alloc scratch): ") + cudaGetErrorString(ce);
      return -1;
    }
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return 0;
}

void set_error(char** err, const std::string& msg) {
  if (err) *err = strdup(msg.c_str());
}

}  // namespace

namespace mb {

// Set-up for this entry point on `device`, run by macboost_prepare: looking up
// the scratch's address loads this file's module on that device, which is
// when the GPU reserves the array, so no no-alloc call is the one that
// reserves it.
int noalloc_setup(int device, std::string& err) {
  if (device < 0 || device >= kMaxDevices) {
    err = "device " + std::to_string(device) + " is out of range for the no-alloc scratch";
    return -1;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device && cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    err = "cannot make device " + std::to_string(device) + " current";
    return -1;
  }
  void* p = nullptr;
  const int rc = scratch_address(device, &p, err);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return rc;
}

}  // namespace mb

// (the .cu files are compiled with hidden visibility; this one is exported)
extern "C" __attribute__((visibility("default"))) int32_t macboost_predict_device_noalloc(void* handle, int32_t device,
                                                   const float* x_dev, int64_t rows,
                                                   int64_t cols, int64_t ld, int32_t layout,
                                                   int32_t kind, void* out_dev, void* stream,
                                                   char** err) {
  if (!handle || !x_dev || !out_dev) {
    set_error(err, "null argument");
    return -1;
  }
  mb::Engine& e = *static_cast<mb::Engine*>(handle);
  if (rows < 0) {
    set_error(err, "rows must be >= 0");
    return -1;
  }
  if (cols != e.model.num_features) {
    set_error(err, "model expects " + std::to_string(e.model.num_features) +
                       " features, got " + std::to_string(cols));
    return -1;
  }
  if (kind < mb::kKindPredict || kind > mb::kKindCli) {
    set_error(err, "unknown output kind " + std::to_string(kind));
    return -1;
  }
  if (layout != 0 && layout != 1) {
    set_error(err, "layout must be 0 (feature-major) or 1 (row-major)");
    return -1;
  }
  if (layout == 0 && ld < rows) {
    set_error(err, "feature-major input needs ld >= rows");
    return -1;
  }
  const int64_t ldt = (rows + 3) / 4 * 4;  // row-major input: stride of its copy
  if (layout == 1 && size_t(ldt) * size_t(cols) * 4 > kRowMajorBytes) {
    set_error(err, "row-major input of " + std::to_string(rows) + " x " + std::to_string(cols) +
                       " values exceeds this entry point's 16 MiB scratch (4,194,304 values); "
                       "split the rows or pass feature-major input");
    return -1;
  }
  if (device < 0 || device >= kMaxDevices) {
    set_error(err, "device " + std::to_string(device) + " is out of range");
    return -1;
  }
  if (rows == 0) return 0;

  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device && cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    set_error(err, "cannot make device " + std::to_string(device) + " current");
    return -1;
  }
  auto restore = [&] {
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
  };
  std::string msg;
  void* base = nullptr;
  if (scratch_address(device, &base, msg) != 0) {
    restore();
    set_error(err, msg);
    return -1;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* status = static_cast<unsigned*>(base);
  // the kernel's chunk counters: zero in a fresh module, left at zero by
  // every launch that used them
  auto* sched = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(base) + 16);
  auto* xt = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kStatusBytes);
  cudaError_t ce = cudaMemsetAsync(status, 0, sizeof(unsigned), s);  // left over from the last call
  int rc = 0;
  if (ce != cudaSuccess) {
    msg = std::string("clearing the status word: ") + cudaGetErrorString(ce);
    rc = -1;
  } else if (layout == 1) {
    ce = mb::launch_transpose(x_dev, rows, int(cols), xt, ldt, s);
    if (ce != cudaSuccess) {
      msg = std::string("transpose launch: ") + cudaGetErrorString(ce);
      rc = -1;
    } else {
      rc = mb::engine_launch_resident(e, device, xt, rows, ldt, true, kind, out_dev, status,
                                      sched, s, msg);
    }
  } else {
    rc = mb::engine_launch_resident(e, device, x_dev, rows, ld, true, kind, out_dev, status,
                                    sched, s, msg);
  }
  if (rc == 0) {
    unsigned word = 0;
    ce = cudaMemcpyAsync(&word, status, sizeof(word), cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) {
      msg = std::string("predict: ") + cudaGetErrorString(ce);
      rc = -1;
    } else if (word != 0) {
      msg = "device " + std::to_string(device) +
            ": forest kernel gave up waiting for a shared-memory transfer (status " +
            std::to_string(word) + ")";
      rc = -1;
    }
  }
  restore();
  if (rc != 0) set_error(err, msg);
  return rc;
}
