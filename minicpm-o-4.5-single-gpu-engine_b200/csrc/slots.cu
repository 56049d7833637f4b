// Steady-state (slot-pool) kernels: the per-(step, block) key/value slot pool and the conv-cache row pool of the
// streaming solve (engine/runtime/dit_fast.py:58-97,189-222: FlashInfer paged K/V with page size 1, conv caches of two
// frames per CFG row, step and block).
//
// K/V pool: bf16 [steps * depth][n_slots][2 H] (K then V of one frame).  The attention kernel's gathered mode reads it
// through each row's slot list; k_kv_scatter writes a window's new keys into their slots after the QKV GEMM.
// Conv pool: bf16 [steps * depth][n_rowslots][2 convs][2 frames][H].  The packed row layout keeps two rows in front of
// every window; k_conv_cache fills them with the row's cached frames of the conv's input (so the causal conv GEMM reads
// [cache | window] as consecutive rows) and writes the last two input frames back as the new cache.
#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kWarps = 8;

// A warp copies n16 16-byte chunks: all of a lane's loads are issued before its stores (up to 8 per lane in flight;
// a plain loop keeps one load-store round trip per chunk).
T2W_DEV void warp_copy16(uint4* __restrict__ dst, const uint4* __restrict__ src, int n16, int lane) {
  constexpr int kMax = 8;
  for (int c0 = 0; c0 < n16; c0 += 32 * kMax) {
    uint4 v[kMax];
#pragma unroll
    for (int j = 0; j < kMax; ++j) {
      const int c = c0 + 32 * j + lane;
      if (c < n16) v[j] = src[c];
    }
#pragma unroll
    for (int j = 0; j < kMax; ++j) {
      const int c = c0 + 32 * j + lane;
      if (c < n16) dst[c] = v[j];
    }
  }
}

// One warp per new token: its K and V (2 H bf16 of the QKV output row) into its pool slot.
__global__ void __launch_bounds__(256) k_kv_scatter(const __nv_bfloat16* __restrict__ qkv, int ld_qkv, int H,
                                                    const int* __restrict__ tok_qrow, const int* __restrict__ tok_slot,
                                                    int n, __nv_bfloat16* __restrict__ pool, int pool_ld) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= n) return;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + (size_t)tok_qrow[i] * ld_qkv + H);
  uint4* dst = reinterpret_cast<uint4*>(pool + (size_t)tok_slot[i] * pool_ld);
  warp_copy16(dst, src, 2 * H / 8, lane);
}

// One warp per CFG row: cached frames -> the two rows before its window in `buf`; then the last two rows of
// [cache | window] -> the row's write slot (read before written, so read slot == write slot keeps the cache).
__global__ void __launch_bounds__(256) k_conv_cache(__nv_bfloat16* __restrict__ buf, int H, const ConvRow* __restrict__ rows,
                                                    int n, __nv_bfloat16* __restrict__ cpool, long long slot_ld) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= n) return;
  const ConvRow r = rows[i];
  const int n16 = H / 8;  // 16-byte chunks of a frame
  const uint4* rd = reinterpret_cast<const uint4*>(cpool + (size_t)r.rd * slot_ld);
  uint4* wr = reinterpret_cast<uint4*>(cpool + (size_t)r.wr * slot_ld);
  uint4* b0 = reinterpret_cast<uint4*>(buf + (size_t)(r.seg_row - 2) * H);
  warp_copy16(b0, rd, 2 * n16, lane);  // frames 0, 1 -> rows seg_row - 2, seg_row - 1
  __syncwarp();
  const uint4* last = reinterpret_cast<const uint4*>(buf + (size_t)(r.seg_row - 2 + r.T) * H);
  warp_copy16(wr, last, 2 * n16, lane);
}

// K / V of every (step, block): slot src[i] -> slot dst[i].  One warp per (sb, pair).
__global__ void __launch_bounds__(256) k_slot_copy(__nv_bfloat16* __restrict__ pool, int pool_ld, long long sb_ld, int n_sb,
                                                   const int* __restrict__ src, const int* __restrict__ dst, int n) {
  const long long i = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= (long long)n * n_sb) return;
  const int sb = (int)(i / n), k = (int)(i - (long long)sb * n);
  const uint4* s = reinterpret_cast<const uint4*>(pool + sb * sb_ld + (size_t)src[k] * pool_ld);
  uint4* d = reinterpret_cast<uint4*>(pool + sb * sb_ld + (size_t)dst[k] * pool_ld);
  for (int c = lane; c < pool_ld / 8; c += 32) d[c] = s[c];
}

// Conv caches of every (step, block): row slot src -> dst, or zeros into dst when src < 0.
__global__ void __launch_bounds__(256) k_rowslot_copy(__nv_bfloat16* __restrict__ cpool, long long slot_ld,
                                                      long long sb_ld, int n_sb, int src, int dst) {
  const int sb = blockIdx.x;
  if (sb >= n_sb) return;
  uint4* d = reinterpret_cast<uint4*>(cpool + sb * sb_ld + (size_t)dst * slot_ld);
  const uint4* s = src >= 0 ? reinterpret_cast<const uint4*>(cpool + sb * sb_ld + (size_t)src * slot_ld) : nullptr;
  for (int c = threadIdx.x; c < slot_ld / 8; c += blockDim.x) d[c] = s ? s[c] : make_uint4(0, 0, 0, 0);
}

// x0 of a solve over library-kept caches: token i's channel c = temp * noise[c][col[i]] (the flow's fixed noise,
// [mel, frames], read at each request's cache length).  One thread per (token, channel), token-major output.
__global__ void __launch_bounds__(256) k_noise_x0(const float* __restrict__ noise, int frames, int mel,
                                                  const int* __restrict__ col, int n, float temp, float* __restrict__ x0) {
  pdl_wait();
  pdl_launch();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n * mel) return;
  const int tok = (int)(i / mel), c = (int)(i - (long long)tok * mel);
  x0[i] = temp * noise[(size_t)c * frames + col[tok]];
}

}  // namespace

int launch_noise_x0(const float* noise, int frames, int mel, const int* col, int n, float temp, float* x0,
                    cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  const long long items = (long long)n * mel;
  cudaError_t e = launch_k(k_noise_x0, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, st, noise, frames, mel, col,
                           n, temp, x0);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

int launch_kv_scatter(const __nv_bfloat16* qkv, int H, const int* tok_qrow, const int* tok_slot, int n,
                      __nv_bfloat16* pool, cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  const unsigned g = (unsigned)((n + kWarps - 1) / kWarps);
  cudaError_t e = launch_k(k_kv_scatter, dim3(g), dim3(256), 0, st, qkv, 3 * H, H, tok_qrow, tok_slot, n, pool, 2 * H);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

int launch_conv_cache(__nv_bfloat16* buf, int H, const ConvRow* rows, int n, __nv_bfloat16* cpool, long long slot_ld,
                      cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  const unsigned g = (unsigned)((n + kWarps - 1) / kWarps);
  cudaError_t e = launch_k(k_conv_cache, dim3(g), dim3(256), 0, st, buf, H, rows, n, cpool, slot_ld);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

int launch_slot_copy(__nv_bfloat16* pool, int pool_ld, long long sb_ld, int n_sb, const int* src, const int* dst, int n,
                     cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  const long long items = (long long)n * n_sb;
  k_slot_copy<<<(unsigned)((items + kWarps - 1) / kWarps), 256, 0, st>>>(pool, pool_ld, sb_ld, n_sb, src, dst, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

int launch_rowslot_copy(__nv_bfloat16* cpool, long long slot_ld, long long sb_ld, int n_sb, int src, int dst,
                        cudaStream_t st) {
  k_rowslot_copy<<<n_sb, 256, 0, st>>>(cpool, slot_ld, sb_ld, n_sb, src, dst);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace t2w
