// noalloc.cu — INT8 quantize of several layers' K/V without any device
// allocation.
//
// Some callers cannot call cudaMalloc: a process whose GPU memory is owned
// entirely by another allocator (a framework's caching allocator that has
// reserved the device, a server running under a fixed memory budget), or a
// caller that must not risk cudaMalloc's device-wide implicit
// synchronisation (this entry point waits for its own stream only).
// nkv_int8_quantize_layers_noalloc serves them: the per-layer job table and
// the non-finite flags the quantize kernel needs live in the file-scope array
// below instead of memory allocated per call.  The caller still provides
// every input and output buffer.
//
// The array is a host-side stand-in in host code, not a device address; the
// device address is looked up on every call with cudaGetSymbolAddress (with
// the caller's device current, so a reset device or another context is
// never handed a stale address) and passed to the kernel.  Every GPU that
// loads this library holds the array until exit.  All calls share it and it
// keeps the last call's contents: a call clears the flags it uses, and a
// per-device mutex held from the first copy to the final stream
// synchronisation serialises the calls of one process on one GPU, whichever
// host threads and streams they come from.
#include <cuda_runtime.h>

#include <cstring>
#include <functional>
#include <mutex>
#include <string>

#include "bank.h"
#include "nkv_kernels.h"
#include "nomas_kv.h"

namespace nkv {
int guarded_call(const std::function<void()>& f);  // abi.cpp
}

namespace {

constexpr int kMaxLayers = NKV_NOALLOC_MAX_LAYERS;
constexpr int kMaxDevices = 64;

struct Scratch {
  nkv::QuantJob jobs[kMaxLayers];
  uint32_t flags[kMaxLayers + 1];  // [0]: any layer; [1 + i]: layer i
};

// 64 layers x 56-byte jobs + flags: about 3.9 KB per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(Scratch)];

std::mutex g_dev_mu[kMaxDevices];

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) nkv::fail(NKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" int nkv_int8_quantize_layers_noalloc(const void* const* k, const void* const* v, int32_t n_layers,
                                                int32_t in_dtype, uint64_t rows, int64_t head_dim,
                                                uint8_t* const* kq, uint8_t* const* vq, float* const* ks,
                                                float* const* vs, uint32_t* nonfinite_out, void* stream) {
  return nkv::guarded_call([&] {
    if (n_layers < 1 || n_layers > kMaxLayers)
      nkv::fail(NKV_ERR_ARGUMENT, "n_layers must be in [1, " + std::to_string(kMaxLayers) + "], got " +
                                      std::to_string(n_layers));
    if (in_dtype < NKV_F32 || in_dtype > NKV_F16) nkv::fail(NKV_ERR_ARGUMENT, "unknown dtype");
    if (head_dim < 1) nkv::fail(NKV_ERR_ARGUMENT, "head_dim must be >= 1");
    if (!k || !v || !kq || !vq || !ks || !vs || !nonfinite_out) nkv::fail(NKV_ERR_ARGUMENT, "null pointer array");
    for (int i = 0; i < n_layers; ++i)
      if (!k[i] || !v[i] || !kq[i] || !vq[i] || !ks[i] || !vs[i])
        nkv::fail(NKV_ERR_ARGUMENT, "null pointer for layer " + std::to_string(i));
    for (int i = 0; i < n_layers; ++i) nonfinite_out[i] = 0;
    if (rows == 0) return;

    int dev = 0;
    cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) nkv::fail(NKV_ERR_ARGUMENT, "device index too large");
    std::lock_guard<std::mutex> lock(g_dev_mu[dev]);
    // The array's device address in the current device's context.
    void* base = nullptr;
    cuda_ok(cudaGetSymbolAddress(&base, g_noalloc_scratch), "cudaGetSymbolAddress");
    Scratch* sc = static_cast<Scratch*>(base);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    nkv::QuantJob host_jobs[kMaxLayers];
    bool aligned = true;
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    for (int i = 0; i < n_layers; ++i) {
      host_jobs[i] = nkv::QuantJob{k[i], v[i], kq[i], vq[i], ks[i], vs[i], &sc->flags[1 + i]};
      aligned &= a16(k[i]) && a16(v[i]) && a16(kq[i]) && a16(vq[i]);
    }
    // The flags keep the previous call's values: clear them before the kernel.
    cuda_ok(cudaMemsetAsync(sc->flags, 0, sizeof(uint32_t) * (n_layers + 1), s), "cudaMemsetAsync");
    cuda_ok(cudaMemcpyAsync(sc->jobs, host_jobs, sizeof(nkv::QuantJob) * n_layers, cudaMemcpyHostToDevice, s),
            "cudaMemcpyAsync");
    cuda_ok(nkv::launch_int8_quantize(sc->jobs, n_layers, rows, 0, head_dim, in_dtype, aligned, sc->flags, s),
            "quantize");
    uint32_t flags[kMaxLayers + 1];
    cuda_ok(cudaMemcpyAsync(flags, sc->flags, sizeof(uint32_t) * (n_layers + 1), cudaMemcpyDeviceToHost, s),
            "cudaMemcpyAsync");
    cuda_ok(cudaStreamSynchronize(s), "quantize");
    for (int i = 0; i < n_layers; ++i) nonfinite_out[i] = flags[1 + i];
    if (flags[0] != 0) {
      int first = 0;
      while (first < n_layers && flags[1 + first] == 0) ++first;
      const bool k_bad = first < n_layers && (flags[1 + first] & 1u) != 0;
      nkv::fail(NKV_ERR_MSG, std::string("cannot quantize non-finite ") + (k_bad ? "k" : "v") + " values");
    }
  });
}
