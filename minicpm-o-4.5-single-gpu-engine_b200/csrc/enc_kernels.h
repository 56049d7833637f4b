// Internal launch interface of the flow-encoder kernels (enc_kernels.cu; not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace t2w {

// One work entry of the relative-position attention: a 128-query tile of one sequence (the window's queries are rows
// q_row .. of the qkv4 buffer, the tile's first query is query q_pos of T; the sequence's K keys are pool rows
// kv_idx[kv_off .. kv_off + K)).  Each entry runs as `heads` CTAs.
struct RelWork {
  int q_row, q_pos, T, K, kv_off;
};
struct RelArgs {
  const RelWork* work = nullptr;  // device [n_work]
  int n_work = 0, heads = 0;
  const __nv_bfloat16* pool = nullptr;  // [pool_rows, 2 heads 64]: [k | v]
  int pool_ld = 0;
  const int* kv_idx = nullptr;
  int r0 = 0;  // table row of relative position 0 (max_frames - 1)
  __nv_bfloat16* out = nullptr;
  int ldo = 0;
  float scale_log2 = 0.f;
  int* err = nullptr;
};
// Tensor maps: tm_q over the qkv4 buffer (bf16 [rows, 4 H], 128-row x 64-column boxes), tm_pos over the
// relative-position table (bf16 [2 max_frames - 1, H], 160-row x 64-column boxes).
bool make_relattn_tmaps(CUtensorMap* tm_q, CUtensorMap* tm_pos, const void* qkv4, int rows, int H, const void* pos,
                        int max_frames);
int launch_relattn(const RelArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_pos, cudaStream_t st);

// pos[row][n] = bf16(sum_k w[n][k] pe(row - (max_frames - 1))[k]), fp32 math.
int launch_pos_table(const float* w, int H, int max_frames, float max_period, __nv_bfloat16* pos, cudaStream_t st);

// Row LayerNorm y = LN(x) w + b (fp32 x; fp32 and / or bf16 outputs; pad rows zero).  C % 128 == 0, C <= 1024.
int launch_enc_ln(const float* x, const float* w, const float* b, float eps, int rows, int C, float* out_f32,
                  __nv_bfloat16* out_bf16, const uint8_t* pad, cudaStream_t st);

// out[r] = emb[tok[r]] (bf16 rows of C), zeros where tok[r] < 0.
int launch_embed_rows(const __nv_bfloat16* emb, const int* tok, int rows, int C, __nv_bfloat16* out, cudaStream_t st);

// A window's rows in the encoder's buffers: its first-stack segment starts at seg1 (2 conv-cache rows, then its frames),
// its second-stack segment at seg2 (2 stride conv-cache rows, then its upsampled frames); T frames; conv-cache row
// `cache` of the [n][2 + 2 stride][C] bf16 cache pool.
struct EncRow {
  int seg1, T, cache, seg2;
};
// Pre-lookahead conv2's cache: rows seg1, seg1 + 1 of o <- the cached frames; the cache <- the last two frames of
// [cache | o's T frames] (one block per window).
int launch_pl_cache(__nv_bfloat16* o, int C, const EncRow* rows, int n, __nv_bfloat16* cache, int cache_frames,
                    cudaStream_t st);
// Upsampling input: u rows seg2 .. seg2 + 3 <- the cached frames, rows seg2 + 4 + 2 t + {0, 1} <- bf16(h[seg1 + 2 + t]);
// the cache <- the last four frames of [cache | upsampled] (one block per window).
int launch_up_pack(const float* h, int C, const EncRow* rows, int n, __nv_bfloat16* u, __nv_bfloat16* cache,
                   int cache_frames, cudaStream_t st);
// pool[slot[i]] <- qkv4[row[i]][2 H .. 4 H) (the new keys' [k | v]).
int launch_enc_kv_scatter(const __nv_bfloat16* qkv4, int H, const int* row, const int* slot, int n, __nv_bfloat16* pool,
                          cudaStream_t st);
// out[i] = src[row[i]] (fp32 rows of C floats).
int launch_gather_rows_f32(const float* src, int C, const int* row, int n, float* out, cudaStream_t st);

}  // namespace t2w
