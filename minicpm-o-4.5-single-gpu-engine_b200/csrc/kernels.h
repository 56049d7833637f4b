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
// The same with a 32-, 64- or 128-byte swizzle (box_cols * elem_bytes == swizzle_bytes).
bool make_tmap_2d_ex(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                     uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols, int swizzle_bytes);

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
  // Completion counters, one per 128-row block: each epilogue warp adds 1 once its stores of a tile are complete
  // (8 per tile; a block is done at 8 * N / BN).  Lets the row kernel that follows start early (RowWait).
  int* done_flags = nullptr;
  // L2 prefetch of the next GEMM's weights, issued by each CTA as its producer starts its last tile (64 KB per CTA)
  const void* pf = nullptr;
  unsigned pf_bytes = 0;
  const float* gate = nullptr;  // T2W_EPI_RESID: out (fp32) += gate[n] * (acc + bias[n]), N floats
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

// Block-scaled FP8 GEMM (gemm8.cu): A8 e4m3 [rows_a, lda bytes] with UE8M0 scale atoms per (128-row tile, 128-column
// block) in `sfa_layouts` row-shifted layouts (layout d at sfa + d * sfa_layout; the causal conv needs d = 0, 1, 2),
// W8 e4m3 [N, taps * K] with atoms [taps * K / 128][N / 128][512].  Epilogues T2W_EPI_BF16, T2W_EPI_QKV (bf16 out)
// and T2W_EPI_GELU_FP8 (e4m3 out with its scale atoms in out_sf, layout 0).
struct Gemm8Args {
  const void* A8 = nullptr;
  int lda = 0, rows_a = 0;
  const uint8_t* sfa = nullptr;
  long long sfa_layout = 0;
  int sfa_layouts = 1;
  const void* W8 = nullptr;
  const uint8_t* sfw = nullptr;
  const float* bias = nullptr;
  int M = 0, N = 0, K = 0, taps = 1, tap_row0 = 0;
  int epi = 0;
  void* out = nullptr;
  int ldo = 0;  // elements of the output type
  uint8_t* out_sf = nullptr;
  const float* qn_w = nullptr;
  const float* qn_b = nullptr;
  const float* kn_w = nullptr;
  const float* kn_b = nullptr;
  float qk_eps = 0.f;
  int* err = nullptr;
  // L2 prefetch of the next GEMM's weights, issued by each CTA as its producer starts its last tile (64 KB per CTA)
  const void* pf = nullptr;
  unsigned pf_bytes = 0;
};
// Bytes of one layout of scale atoms for a [rows, cols] e4m3 matrix.
size_t gemm8_sf_bytes(int rows, int cols);
// tmA / tmW / tmC may be prebuilt (A: 128 x 128-byte boxes; W: 256 x 128; C: 32-row boxes of 64 bf16 columns with
// 128-byte swizzle, or of 64 e4m3 columns with 64-byte swizzle).
int launch_gemm8(const Gemm8Args& a, cudaStream_t st, const CUtensorMap* tmA = nullptr, const CUtensorMap* tmW = nullptr,
                 const CUtensorMap* tmC = nullptr);

// One attention work item: a 128-query tile of one packed sequence (gathered form: k_row is the offset of the row's
// key list in kv_idx, P its window's query count, L its key count).
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
  void* out = nullptr;  // bf16 [rows, heads * 64], or e4m3 when out_sf is set
  uint8_t* out_sf = nullptr;  // e4m3 output: its UE8M0 scale atoms (layout 0)
  float scale_log2 = 0.f;
  // Gathered keys (slot-pool form; pool != nullptr): work item keys j = pool rows kv_idx[k_row + j], K at column
  // h * 64 and V at heads * 64 + h * 64 of rows of pool_ld bf16; the item's P queries (from q_pos) see all L keys.
  const __nv_bfloat16* pool = nullptr;
  const int* kv_idx = nullptr;
  int pool_ld = 0;
  int* err = nullptr;
  const void* pf = nullptr;  // L2 prefetch of the next GEMM's weights (64 KB per CTA of the first CTAs)
  unsigned pf_bytes = 0;
  // Paired form (gathered keys only): two (query tile, head) items share each 128-row MMA tile, block-diagonally.
  // Every work item's queries must lie within 64 rows (P - q_pos <= 64); rows past 64 would not be computed, so the
  // caller checks this on its host copy of the work list.  tm_q_pair: the query map with 64-row boxes
  // (make_attn_pair_tmap), or nullptr to make one per launch.
  bool pair = false;
  const CUtensorMap* tm_q_pair = nullptr;
};
// Tensor maps of the attention kernel over a qkv buffer: 128-row query boxes and 64-row key / value boxes.
bool make_attn_tmaps(CUtensorMap* tm_q, CUtensorMap* tm_kv, const void* qkv, int rows, int heads);
// The paired form's query map: 64-row boxes.
bool make_attn_pair_tmap(CUtensorMap* tm_q, const void* qkv, int rows, int heads);
int launch_attn(const AttnArgs& a, cudaStream_t st, const CUtensorMap* tm_q = nullptr, const CUtensorMap* tm_kv = nullptr);

// Slot-pool (steady-state) kernels, slots.cu.  A conv row: a CFG row's window starts at buffer row seg_row (its two
// cache rows sit just before it), has T frames, reads conv-cache row slot rd and writes rd's new frames to wr.
struct ConvRow {
  int seg_row, T, rd, wr;
};
int launch_kv_scatter(const __nv_bfloat16* qkv, int H, const int* tok_qrow, const int* tok_slot, int n,
                      __nv_bfloat16* pool, cudaStream_t st);
// cpool: this (step, block)'s conv pool at the conv's frames of row slot 0; slot_ld: elements between row slots.
int launch_conv_cache(__nv_bfloat16* buf, int H, const ConvRow* rows, int n, __nv_bfloat16* cpool, long long slot_ld,
                      cudaStream_t st);
int launch_slot_copy(__nv_bfloat16* pool, int pool_ld, long long sb_ld, int n_sb, const int* src, const int* dst, int n,
                     cudaStream_t st);
int launch_rowslot_copy(__nv_bfloat16* cpool, long long slot_ld, long long sb_ld, int n_sb, int src, int dst,
                        cudaStream_t st);
// x0[i][c] = temp * noise[c * frames + col[i]] for n tokens (token-major [n, mel] fp32).
int launch_noise_x0(const float* noise, int frames, int mel, const int* col, int n, float temp, float* x0,
                    cudaStream_t st);

// Row kernels.
int launch_ln_mod(const float* h, int ldh, const float* shift, const float* scale1, float eps, int rows, int C,
                  __nv_bfloat16* out, int ldo, const uint8_t* pad, cudaStream_t st);
// Output of a row kernel: bf16 [rows, C], or e4m3 [rows, C] with UE8M0 scale atoms per (row, 32-column block) written
// in n_layouts row-shifted layouts (layout d at sf + d * layout_bytes holds row x at position x + d: d = 0 for a plain
// GEMM operand, d = 0, 1, 2 for the causal conv's taps).
struct RowOut {
  void* out = nullptr;
  uint8_t* sf = nullptr;
  int n_layouts = 1;
  long long layout_bytes = 0;
};
inline RowOut row_out_bf16(__nv_bfloat16* p) {
  RowOut o;
  o.out = p;
  return o;
}
// A row kernel that follows a GEMM with done_flags: instead of waiting for the GEMM's whole grid (programmatic launch)
// each warp waits until its row's 128-row block reached `target` (bounded; T2W_ERR_TIMEOUT into err), so the rows of
// finished tiles are normalised on SMs the GEMM's last partial wave leaves idle.  flags == nullptr: plain ordering.
struct RowWait {
  const int* flags = nullptr;
  int target = 0;
  int* err = nullptr;
  // L2 prefetch of the next GEMM's weights, issued as the kernel starts (64 KB per block of the first blocks)
  const void* pf = nullptr;
  unsigned pf_bytes = 0;
  const void* pf2 = nullptr;
  unsigned pf2_bytes = 0;
  // the wait's limit in ns (0: the library's 2 s); a shorter one lets a test make a wait run out quickly
  unsigned long long limit_ns = 0;
};
// h += g * y (fp32, in place; skipped when y == nullptr), then out = LN(h) * scale1 + shift, pad rows zero.
int launch_add_ln_mod(float* h, const __nv_bfloat16* y, const float* g, const float* shift, const float* scale1, float eps,
                      int rows, int C, const RowOut& o, const uint8_t* pad, cudaStream_t st, const RowWait& wt = RowWait());
int launch_ln_mish(const __nv_bfloat16* x, const float* w, const float* b, float eps, int rows, int C, const RowOut& o,
                   const uint8_t* pad, cudaStream_t st, const RowWait& wt = RowWait());
// bf16 [rows, C] -> e4m3 + scale atoms (C = 128, 512, 1536 or 2048).
int launch_quant_rows(const __nv_bfloat16* x, int rows, int C, const RowOut& o, cudaStream_t st);
// fp32 W [N, Kt] -> e4m3 + per-1x128-block scale atoms [Kt / 128][N / 128][512].
int launch_quant_weight(const float* w, int N, int Kt, uint8_t* w8, uint8_t* sf, cudaStream_t st);
// Conv1d weight [out, in, k] fp32 -> fp32 [out, k * in], tap-major (the FP8 path quantises this layout).
int launch_conv_weight_f32(const float* src, float* dst, int cout, int cin, int k, cudaStream_t st);
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
