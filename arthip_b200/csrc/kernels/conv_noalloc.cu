// Allocation-free variant of the tensor-core 3x3 conv layer (ah_conv3x3_run_noalloc).
//
// Who needs it: callers that cannot allocate GPU memory at the point they run a layer,
// e.g. a plugin host that hands its plugins device buffers from its own pool and forbids
// cudaMalloc inside the plugin (a cudaMalloc there can block on a device-wide
// synchronisation, or fail once the host has budgeted all of the GPU's memory).
//
// The regular entry point (ah_conv3x3_create/run) keeps the packed weights, the fp32 bias
// and the kernel's error word in device memory it allocates at create time. This variant
// keeps the same three in one file-scope __device__ array of fixed size instead, so a call
// allocates nothing: the caller passes the input, optional residual tensors and output,
// and the weights as host fp16 bits on every call.
//
// Limits and sharing:
//  * the array holds kNoAllocWeightBytes of packed weights, which covers every layer the
//    tensor-core kernel supports (C % 16 == 0, C <= 128, M <= 256); every GPU on which the
//    library's device code is loaded holds the whole array until the process exits;
//  * every call on a device shares that device's array and leaves the last call's weights
//    in it; the error word is cleared at the start of each call. Calls whose GPU work
//    overlaps on one device (other host threads, or other streams) would race on the array
//    and give wrong results, so calls on one device are serialised on the host and each
//    call returns only after its kernel has finished. Calls on different devices run
//    concurrently; they share only the host staging buffer, held while it is packed and
//    copied;
//  * each call looks up the array's device address (cudaGetSymbolAddress, which allocates
//    nothing) with the device current, so a device reset between calls is harmless;
//  * `stream` must belong to `device` (checked); the caller's current device is restored
//    on return.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../../include/arthip_b200.h"
#include "kernels.h"

namespace ah {
namespace {
// Largest packed weight image: 9 taps x 256 output channels x 128 input channels x 2 bytes.
constexpr size_t kNoAllocWeightBytes = static_cast<size_t>(9) * 256 * 128 * 2;
constexpr size_t kNoAllocBiasOff = kNoAllocWeightBytes;             // 256 fp32 (Mpad <= 256)
constexpr size_t kNoAllocStatusOff = kNoAllocBiasOff + 256 * sizeof(float);
constexpr size_t kNoAllocScratchBytes = kNoAllocStatusOff + 256;
constexpr int kNoAllocMaxDevices = 64;
}  // namespace
}  // namespace ah

// The scratch array (file scope). In host code `g_noalloc_scratch` names a host-side
// stand-in, not the device memory: kernels are given the address that
// cudaGetSymbolAddress returns for the current device (scratch_base below).
static __device__ __align__(256) uint8_t g_noalloc_scratch[ah::kNoAllocScratchBytes];

namespace ah {
namespace {

// Host staging of the packed weights and bias (static storage: no heap either), shared by
// all devices and guarded by g_host_mu while a call packs and copies it.
alignas(64) uint8_t g_pack_host[kNoAllocWeightBytes];
float g_bias_host[256];

std::mutex g_host_mu;                        // the staging arrays above
std::mutex g_dev_mu[kNoAllocMaxDevices];     // one call at a time per device (its array)

void copy_err(const std::string& s, char* dst, int len) {
  if (!dst || len <= 0) return;
  size_t n = s.size();
  if (n > static_cast<size_t>(len) - 1) n = static_cast<size_t>(len) - 1;
  std::memcpy(dst, s.data(), n);
  dst[n] = '\0';
}

// Device address of the array on the current device. Called on every call, with the
// call's device current.
cudaError_t scratch_base(uint8_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<uint8_t*>(p);
  return cudaSuccess;
}

// Restores the caller's current device when the call returns.
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      prev = -1;
      (void)cudaGetLastError();
    }
  }
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

}  // namespace ah

extern "C" int ah_conv3x3_run_noalloc(int device, int C, int M, const uint16_t* w_oihw_f16, const float* bias,
                                      int act, const void* in_nhwc, int H, int W, const void* add1,
                                      const void* add2, void* out_nhwc, void* stream, char* err, int errlen) {
  using namespace ah;
  if (!w_oihw_f16 || !in_nhwc || !out_nhwc || H <= 0 || W <= 0 || C <= 0 || M <= 0 || act < 0 || act > 2) {
    copy_err("invalid no-alloc conv arguments", err, errlen);
    return 1;
  }
  if (C % 16 != 0 || C > 128 || M > 256) {
    copy_err("no-alloc conv supports C % 16 == 0, C <= 128 and M <= 256 (got C=" + std::to_string(C) +
                 ", M=" + std::to_string(M) + ")",
             err, errlen);
    return 1;
  }
  if (device < 0 || device >= kNoAllocMaxDevices) {
    copy_err("no-alloc conv: device index out of range", err, errlen);
    return 1;
  }
  DeviceRestore restore;
  std::lock_guard<std::mutex> dev_lock(g_dev_mu[device]);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    copy_err(std::string("cudaSetDevice(") + std::to_string(device) + ") failed: " + cudaGetErrorString(e), err,
             errlen);
    (void)cudaGetLastError();
    return 1;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int sdev = device;
  e = cudaStreamGetDevice(s, &sdev);
  if (e != cudaSuccess || sdev != device) {
    copy_err(e != cudaSuccess ? std::string("no-alloc conv: invalid stream: ") + cudaGetErrorString(e)
                              : "no-alloc conv: the stream belongs to device " + std::to_string(sdev) +
                                    ", not device " + std::to_string(device),
             err, errlen);
    (void)cudaGetLastError();
    return 1;
  }
  uint8_t* base = nullptr;
  e = scratch_base(&base);
  if (e != cudaSuccess) {
    copy_err(std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") + cudaGetErrorString(e), err,
             errlen);
    (void)cudaGetLastError();
    return 1;
  }

  ConvTcWeights L;
  const size_t bytes = conv_tc_pack_layout(C, M, &L);
  if (bytes > kNoAllocWeightBytes) {
    copy_err("no-alloc conv: packed weights (" + std::to_string(bytes) + " bytes) exceed the " +
                 std::to_string(kNoAllocWeightBytes) + "-byte scratch",
             err, errlen);
    return 1;
  }
  L.wpack = base;
  L.bias = reinterpret_cast<float*>(base + kNoAllocBiasOff);
  uint32_t* status = reinterpret_cast<uint32_t*>(base + kNoAllocStatusOff);

  ConvTcOut to;
  to.ptr = out_nhwc;
  to.mode = (M % 16 == 0) ? 0 : 1;
  ConvTcPlan plan;
  std::string perr;
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) sms = 148;
  if (!conv_tc_plan(&L, static_cast<const __half*>(in_nhwc), H, W, to, sms, &plan, &perr)) {
    copy_err(perr, err, errlen);
    return 1;
  }
  // Stream-ordered: weights, bias and a cleared error word, then the kernel, then the word
  // back. The host copies are from pageable memory, so each copy call returns once the
  // staging arrays have been read (they are free for another device's call then); the final
  // synchronisation makes the call complete on return.
  {
    std::lock_guard<std::mutex> host_lock(g_host_mu);
    conv_tc_pack_into(w_oihw_f16, L, g_pack_host);
    for (int m = 0; m < L.Mpad; ++m) g_bias_host[m] = (bias && m < M) ? bias[m] : 0.f;
    e = cudaMemcpyAsync(base, g_pack_host, bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(L.bias, g_bias_host, sizeof(float) * L.Mpad, cudaMemcpyHostToDevice, s);
  }
  if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess)
    e = conv_tc_launch(plan, static_cast<const __half*>(add1), static_cast<const __half*>(add2), act, status, s);
  uint32_t word = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&word, status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    copy_err(std::string("no-alloc conv failed: ") + cudaGetErrorString(e), err, errlen);
    (void)cudaGetLastError();
    return 2;
  }
  if (word != 0) {
    copy_err("tensor-core conv kernel reported a timed-out pipeline wait (status " + std::to_string(word) + ")", err,
             errlen);
    return 2;
  }
  return 0;
}
