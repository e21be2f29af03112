// Internal launch interface shared by the kernels and the C ABI (gdn_capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace gdn {

enum DType : int { kFP32 = 0, kBF16 = 1 };
enum Semantics : int { kExact = 0, kReference = 1 };

struct RecurrentArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* hT;
  int B, T, H, dk, dv, dtype;
  int Hk;  // heads of q and k (H % Hk == 0); value head h reads q/k head h * Hk / H
};

struct ChunkArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* hT;
  int B, T, H, dk, dv, chunk, dtype, semantics;
  void* workspace;
  size_t ws_bytes;
  int Hk;  // heads of q and k (H % Hk == 0); value head h reads q/k head h * Hk / H
  // Packed variable-length sequences: B sequences in one row of T tokens, sequence s
  // being tokens [cu_seqlens[s], cu_seqlens[s + 1]) (device array of B + 1); NULL: dense.
  const int* cu_seqlens = nullptr;
};

cudaError_t launch_recurrent(const RecurrentArgs& a, cudaStream_t st);

// Decode step (T == 1) with the state streamed by bulk copies (dk = dv = 128).
bool recurrent_bulk_supported(const RecurrentArgs& a);
cudaError_t launch_recurrent_bulk(const RecurrentArgs& a, cudaStream_t st);

// Device error words of the kernel files with bounded waits (0 = none).
int device_error_recurrent_bulk(bool clear);
int device_error_chunk_tc(bool clear);

// Tensor-core chunk kernel: bf16, dk = 128, dv % 64 == 0, chunk = 64, exact.
bool chunk_tc_supported(const ChunkArgs& a);
cudaError_t launch_chunk_tc(const ChunkArgs& a, cudaStream_t st);

// Portable CUDA-core chunk kernel (any supported shape, fp32 or bf16 inputs).
cudaError_t launch_chunk_simt(const ChunkArgs& a, cudaStream_t st);
// Shared-memory bytes launch_chunk_simt needs for this shape (0 = unsupported).
size_t chunk_simt_smem_bytes(const ChunkArgs& a);

}  // namespace gdn
