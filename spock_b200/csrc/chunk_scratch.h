// Per-context device scratch for the chunk-prefill path: fp16 copies of
// q, k, v when the caller's inputs are fp32 or ask for in-kernel L2
// normalisation (the tensor-core kernel reads fp16/bf16 tiles by TMA).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace spock {
struct ChunkScratch {
  void* buf = nullptr;
  size_t bytes = 0;
  // Grows the buffer to at least n bytes. cudaFree of an old buffer waits for
  // the device to go idle, so a buffer still read by queued work is never freed.
  cudaError_t reserve(size_t n) {
    if (n <= bytes) return cudaSuccess;
    if (buf) cudaFree(buf);
    buf = nullptr;
    bytes = 0;
    cudaError_t e = cudaMalloc(&buf, n);
    if (e == cudaSuccess) bytes = n;
    return e;
  }
  void release() {
    if (buf) cudaFree(buf);
    buf = nullptr;
    bytes = 0;
  }
};
}  // namespace spock
