// KV block swap between the paged device pool and a pinned host pool (offload preemption).
//
// The device pool is [cache_layers][2 (K, V)][kv_rows][row_bytes]: block b of one (layer, K/V)
// plane is block_size consecutive rows, so a block over the whole cache is `planes` equal chunks
// spaced one plane apart. A host block stores the same chunks back to back:
// [host_blocks][planes][block_size * row_bytes]. Each block therefore moves as one 2-D copy
// (width = one chunk, height = planes, device pitch = one plane), queued on the caller's stream
// so it is ordered with the launches that wrote the rows and with those that reuse the blocks.
// Copies only: no kernel runs, and every block id is checked on the host before any copy is queued.
#include "cdb_common.cuh"
#include "cdb_b200.h"

extern "C" int cdb_kv_blocks_host_copy(void* kv_base, int num_cache_layers, int64_t kv_rows, int64_t row_bytes,
                                       int block_size, int num_device_blocks, const int32_t* device_blocks,
                                       void* host_pool, int num_host_blocks, const int32_t* host_blocks, int num,
                                       int to_host, void* stream) {
  if (kv_base == nullptr || host_pool == nullptr || num_cache_layers <= 0 || row_bytes <= 0 || block_size <= 0 ||
      num < 0 || num_device_blocks <= 0 || num_host_blocks <= 0 ||
      (int64_t)num_device_blocks * block_size > kv_rows)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num == 0) return CDB_OK;
  if (device_blocks == nullptr || host_blocks == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < num; ++i) {
    if (device_blocks[i] < 0 || device_blocks[i] >= num_device_blocks || host_blocks[i] < 0 ||
        host_blocks[i] >= num_host_blocks)
      return CDB_ERR_INDEX;
  }
  const size_t planes = 2 * (size_t)num_cache_layers;
  const size_t chunk = (size_t)block_size * (size_t)row_bytes;
  const size_t plane_pitch = (size_t)kv_rows * (size_t)row_bytes;
  int dev = 0;
  int max_pitch = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&max_pitch, cudaDevAttrMaxPitch, dev) != cudaSuccess)
    return CDB_ERR_CUDA;
  const bool two_d = plane_pitch <= (size_t)max_pitch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* kv = static_cast<char*>(kv_base);
  char* host = static_cast<char*>(host_pool);
  for (int i = 0; i < num; ++i) {
    char* d = kv + (size_t)device_blocks[i] * chunk;
    char* h = host + (size_t)host_blocks[i] * planes * chunk;
    cudaError_t e = cudaSuccess;
    if (two_d) {
      e = to_host ? cudaMemcpy2DAsync(h, chunk, d, plane_pitch, chunk, planes, cudaMemcpyDeviceToHost, s)
                  : cudaMemcpy2DAsync(d, plane_pitch, h, chunk, chunk, planes, cudaMemcpyHostToDevice, s);
    } else {
      // planes further apart than a 2-D copy's pitch limit: one copy per plane
      for (size_t p = 0; p < planes && e == cudaSuccess; ++p) {
        e = to_host ? cudaMemcpyAsync(h + p * chunk, d + p * plane_pitch, chunk, cudaMemcpyDeviceToHost, s)
                    : cudaMemcpyAsync(d + p * plane_pitch, h + p * chunk, chunk, cudaMemcpyHostToDevice, s);
      }
    }
    if (e != cudaSuccess) return CDB_ERR_CUDA;
  }
  return CDB_OK;
}
