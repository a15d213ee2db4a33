// t5e_noalloc.cu -- evaluation of a host-resident batch that allocates no
// memory, for callers that cannot allocate on the GPU.
//
// Some callers cannot call cudaMalloc or any other allocator: a plugin
// loaded into a host application that owns every GPU memory pool and forbids
// its plugins to allocate; a latency-critical loop that must not allocate
// once it runs (an allocation can block on the device or fail under memory
// pressure); a process held to a fixed GPU memory budget.  They hold their
// batch in host memory.  t5e_mma_dot_batch_noalloc stages that batch in one
// file-scope device array instead of memory it would allocate: the array
// takes T5E_NOALLOC_STAGE_BYTES on every GPU that loads the library, from
// load until the process exits, and every call on a GPU shares it.
//
// Host code cannot use the array's name as a device address, so the
// device address is looked up once per device with cudaGetSymbolAddress
// (with that device current) and kept.  Every call synchronizes its stream,
// so a call on a capturing stream is refused before anything is queued.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "t5e.h"
#include "t5e_dispatch.h"

namespace t5e {
namespace noalloc {

// The staging array: operand rows, C words, scales, metadata, result words
// and status bytes of one batch, each region starting on a 256-byte
// boundary.
static __device__ __align__(256) uint8_t g_stage[T5E_NOALLOC_STAGE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
uint8_t* g_stage_addr[kMaxDevices] = {};  // device address of g_stage, per device, once looked up

int stage_address(int dev, uint8_t*& out) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_cuda_error("t5e_mma_dot_batch_noalloc: device ordinal out of range", cudaErrorInvalidDevice);
    return T5E_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_stage_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_stage);  // `dev` is the current device
    if (e != cudaSuccess) {
      set_cuda_error("t5e_mma_dot_batch_noalloc: cudaGetSymbolAddress of the staging array", e);
      return T5E_ERR_CUDA;
    }
    g_stage_addr[dev] = static_cast<uint8_t*>(p);
  }
  out = g_stage_addr[dev];
  return T5E_OK;
}

uint64_t round256(uint64_t x) { return (x + 255u) & ~uint64_t(255); }

}  // namespace noalloc
}  // namespace t5e

extern "C" int t5e_mma_dot_batch_noalloc(const t5e_model* model, const t5e_batch* host, void* stream) {
  using namespace t5e;
  using namespace t5e::noalloc;
  // the same checks as t5e_mma_dot_batch, on the host geometry, before any
  // CUDA call
  const int v = validate(model, host);
  if (v != T5E_OK) return v;
  if (host->tile_m != 1 || host->tile_n != 1) return T5E_ERR_INVALID;
  const uint64_t n = host->n;
  if (n == 0) return T5E_OK;
  const bool sparse = host->sparse != 0;
  const bool broadcast = sparse && (host->flags & T5E_META_BROADCAST);
  const bool scaled = host->nscale > 0 && host->scale_a && host->scale_b;
  const uint64_t cap = T5E_NOALLOC_STAGE_BYTES;
  char message[160];
  // every factor is at most 2**25 before a product is formed, so no product overflows
  if (n > cap || (uint64_t)host->a_stride > cap || (uint64_t)host->b_stride > cap ||
      (scaled && (uint64_t)host->nscale > cap) || (sparse && (uint64_t)host->meta_words > cap)) {
    std::snprintf(message, sizeof message, "t5e_mma_dot_batch_noalloc: batch larger than the %llu-byte staging array",
                  (unsigned long long)cap);
    set_cuda_error(message, cudaErrorInvalidValue);
    return T5E_ERR_INVALID;
  }
  const uint64_t a_bytes = n * (uint64_t)host->a_stride, b_bytes = n * (uint64_t)host->b_stride;
  const uint64_t c_bytes = n * (uint64_t)host->c_bytes;
  const uint64_t s_bytes = scaled ? n * (uint64_t)host->nscale : 0;
  const uint64_t m_bytes = sparse ? (broadcast ? 1 : n) * (uint64_t)host->meta_words * 4 : 0;
  const uint64_t d_bytes = n * 4, st_bytes = host->status ? n : 0;
  const uint64_t off_b = round256(a_bytes), off_c = off_b + round256(b_bytes), off_sa = off_c + round256(c_bytes);
  const uint64_t off_sb = off_sa + round256(s_bytes), off_m = off_sb + round256(s_bytes);
  const uint64_t off_d = off_m + round256(m_bytes), off_st = off_d + round256(d_bytes);
  const uint64_t need = off_st + round256(st_bytes);
  if (need > cap) {
    std::snprintf(message, sizeof message,
                  "t5e_mma_dot_batch_noalloc: batch needs %llu bytes of staging, more than the %llu-byte array",
                  (unsigned long long)need, (unsigned long long)cap);
    set_cuda_error(message, cudaErrorInvalidValue);
    return T5E_ERR_INVALID;
  }
  // every call ends by synchronizing the stream, which a stream capture does
  // not allow: refuse a capturing stream before anything is queued
  {
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &capture) != cudaSuccess ||
        capture != cudaStreamCaptureStatusNone) {
      set_cuda_error("t5e_mma_dot_batch_noalloc: the stream is capturing (or its state is unknown); the call "
                     "synchronizes its stream and cannot be part of a CUDA graph",
                     cudaErrorStreamCaptureUnsupported);
      return T5E_ERR_INVALID;
    }
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error("t5e_mma_dot_batch_noalloc: cudaGetDevice", e);
    return T5E_ERR_CUDA;
  }
  uint8_t* base = nullptr;
  const int rc_addr = stage_address(dev, base);
  if (rc_addr != T5E_OK) return rc_addr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // everything runs in order on `stream`: the copies up, the cleared result
  // region, the kernel, the copies down
  auto up = [&](uint64_t off, const void* src, uint64_t bytes) {
    return bytes ? cudaMemcpyAsync(base + off, src, bytes, cudaMemcpyHostToDevice, s) : cudaSuccess;
  };
  e = up(0, host->a, a_bytes);
  if (e == cudaSuccess) e = up(off_b, host->b, b_bytes);
  if (e == cudaSuccess) e = up(off_c, host->c, c_bytes);
  if (e == cudaSuccess && scaled) e = up(off_sa, host->scale_a, s_bytes);
  if (e == cudaSuccess && scaled) e = up(off_sb, host->scale_b, s_bytes);
  if (e == cudaSuccess && sparse) e = up(off_m, host->metadata, m_bytes);
  // the array keeps the previous call's words: clear the result region so
  // that no word of an earlier batch can come back
  if (e == cudaSuccess) e = cudaMemsetAsync(base + off_d, 0, d_bytes, s);
  if (e == cudaSuccess && st_bytes) e = cudaMemsetAsync(base + off_st, 0, st_bytes, s);
  if (e != cudaSuccess) {
    set_cuda_error("t5e_mma_dot_batch_noalloc: staging copy", e);
    // copies queued before the failing one may still read the caller's
    // buffers and write the shared array, which the next call reuses
    cudaStreamSynchronize(s);
    return T5E_ERR_CUDA;
  }
  t5e_batch dev_batch = *host;
  dev_batch.a = base;
  dev_batch.b = base + off_b;
  dev_batch.c = base + off_c;
  dev_batch.scale_a = scaled ? base + off_sa : nullptr;
  dev_batch.scale_b = scaled ? base + off_sb : nullptr;
  dev_batch.metadata = sparse ? reinterpret_cast<const uint32_t*>(base + off_m) : nullptr;
  dev_batch.d = reinterpret_cast<uint32_t*>(base + off_d);
  dev_batch.status = host->status ? base + off_st : nullptr;
  const int rc = t5e_mma_dot_batch(model, &dev_batch, stream);
  if (rc != T5E_OK) {
    cudaStreamSynchronize(s);  // the copies above read the caller's buffers
    return rc;
  }
  e = cudaMemcpyAsync(host->d, base + off_d, d_bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && st_bytes) e = cudaMemcpyAsync(host->status, base + off_st, st_bytes, cudaMemcpyDeviceToHost, s);
  // every path returns with this call's copies and kernel finished
  const cudaError_t e_sync = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = e_sync;
  if (e != cudaSuccess) {
    set_cuda_error("t5e_mma_dot_batch_noalloc: result copy", e);
    return T5E_ERR_CUDA;
  }
  return T5E_OK;
}
