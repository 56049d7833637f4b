// Internal host-side launch interface of the Token2Wav kernels (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace t2w {

// Thread-local last CUDA error for t2w_last_cuda_error().
void set_cuda_error(cudaError_t e);
int num_sms();
// Whether kernels are launched with programmatic dependent launch (default on; T2W_PDL=0 turns it off).
bool pdl_enabled();

// Launch `kernel` on `st`, with programmatic stream serialization when enabled.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// TMA tensor map of a row-major 2D bf16 / fp8 matrix [rows, cols] with row pitch `pitch_bytes`, box
// [box_rows, box_cols] (box_cols * elem_bytes == 128: one 128-byte swizzle span), 128-byte swizzle, zero OOB fill.
bool make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                  uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols);

struct GemmArgs {
  const void* A = nullptr;  // bf16 [rows_a, lda]
  int lda = 0, rows_a = 0;
  const void* W = nullptr;  // bf16 [N, taps * K]
  const float* bias = nullptr;
  int M = 0, N = 0, K = 0, taps = 1, tap_row0 = 0;
  int epi = 0;
  void* out = nullptr;
  int ldo = 0;
  const float* qn_w = nullptr;
  const float* qn_b = nullptr;
  const float* kn_w = nullptr;
  const float* kn_b = nullptr;
  float qk_eps = 0.f;
  int* err = nullptr;
};
// Column tile the launcher picks for an N-wide output of M rows with epilogue `epi` (0: N unsupported).
int gemm_block_n_for(int N, int M, int epi);
// Whether some (M, epi) can use an N-wide output at all.
bool gemm_n_supported(int N);
// Tensor maps of one weight matrix W [N, Ktot] bf16 for every column tile the launcher may pick.
struct WeightMaps {
  CUtensorMap bn80, bn128, bn256;
  bool has80 = false, has128 = false, has256 = false;
};
bool make_weight_maps(WeightMaps* m, const void* W, int N, int Ktot);
// Enqueue C = A W^T (+ epilogue).  tmA / W maps / tmC may be prebuilt (nullptr: encoded here; tmC is the output map
// with 128-row boxes of 128 bytes).  Returns a T2W status.
int launch_gemm(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA = nullptr, const WeightMaps* wm = nullptr,
                const CUtensorMap* tmC = nullptr);

// One attention work item: a 128-query tile of one packed sequence.
struct AttnWork {
  int q_row;   // buffer row of the tile's first query
  int k_row;   // buffer row of the sequence's first key
  int q_pos;   // position of the tile's first query in its sequence
  int P, L;    // prompt length, sequence length
};
struct AttnArgs {
  const void* qkv = nullptr;  // bf16 [rows, 3 * heads * 64]
  int rows = 0, heads = 0;
  const AttnWork* work = nullptr;  // device [n_work]
  int n_work = 0;
  void* out = nullptr;  // bf16 [rows, heads * 64]
  float scale_log2 = 0.f;
  int* err = nullptr;
};
// Tensor maps of the attention kernel over a qkv buffer: 128-row query boxes and 64-row key / value boxes.
bool make_attn_tmaps(CUtensorMap* tm_q, CUtensorMap* tm_kv, const void* qkv, int rows, int heads);
int launch_attn(const AttnArgs& a, cudaStream_t st, const CUtensorMap* tm_q = nullptr, const CUtensorMap* tm_kv = nullptr);

// Row kernels.
int launch_ln_mod(const float* h, int ldh, const float* shift, const float* scale1, float eps, int rows, int C,
                  __nv_bfloat16* out, int ldo, const uint8_t* pad, cudaStream_t st);
// h += g * y (fp32, in place; skipped when y == nullptr), then out = bf16(LN(h) * scale1 + shift), pad rows zero.
int launch_add_ln_mod(float* h, const __nv_bfloat16* y, const float* g, const float* shift, const float* scale1, float eps,
                      int rows, int C, __nv_bfloat16* out, const uint8_t* pad, cudaStream_t st);
int launch_ln_mish(const __nv_bfloat16* x, const float* w, const float* b, float eps, int rows, int C,
                   __nv_bfloat16* out, const uint8_t* pad, cudaStream_t st);
int launch_pack(const float* x0, const float* mu, const float* cond, const float* spk, const int* tok_row,
                const int* tok_stream, int n_tok, int mel, int half_rows, __nv_bfloat16* hx, int ld_hx, float* x,
                cudaStream_t st);
int launch_euler(float* x, const float* dphi, int ld_dphi, const int* tok_row, int n_tok, int mel, int half_rows,
                 float dt, float w, __nv_bfloat16* hx, int ld_hx, float* out, cudaStream_t st);
int launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, long long n, cudaStream_t st);
// Conv1d weight [out, in, k] fp32 -> bf16 [out, k * in] (tap-major K: column tap * in + c multiplies frame t - (k-1) + tap).
int launch_conv_weight(const float* src, __nv_bfloat16* dst, int cout, int cin, int k, cudaStream_t st);
// Time embedding MLP + every adaLN modulation table (once per solver).
int launch_temb_mods(const float* ts, int steps, const float* freqs, int freq_dim, float t_scale, const float* fc1_w,
                     const float* fc1_b, const float* fc2_w, const float* fc2_b, int H, const float* const* ada_w,
                     const float* const* ada_b, int depth, const float* fin_w, const float* fin_b, float* silu_temb,
                     float* mods, float* final_mods, cudaStream_t st);

}  // namespace t2w
