// The flow-encoder runtime and its C ABI (t2w_encoder_*, t2w_enc_*, t2w_encode).
//
// An encoder owns its weights (cast to bf16 once, convolutions re-laid out tap-major), a relative-position table per
// conformer layer (linear_pos of the sinusoid at every relative position, computed once in fp32), a K/V key pool per
// layer and a conv-cache row per stream.  The reference keeps each stream's caches as tensors (flow_cache
// conformer_att_cache [d1 + d2, 1, heads, time, 2 d_k] and conformer_cnn_cache [1, C, 6],
// engine/runtime/token2wav_batch.py:408-444) and left-pads them to a common length per call; here a stream is a
// handle whose first- and second-stack caches are ordered lists of pool slots (each layer of a stack stores its keys
// in the same slot of its own pool), so a call needs no padding, no masks and no cache copies: a window's new keys are
// scattered into fresh slots, attention gathers each window's list, and the trim after the call only edits the lists.
//
// One call (t2w_encode) runs every window of the batch together, each with its own token count, cache length and
// final flag.  Row layout (stack 1, one segment per window, T = its frames): [2 conv-cache rows | T frames | 3 look-ahead
// or zero frames]; stack 2: [4 conv-cache rows | 2 T upsampled frames].  The cache rows in front of each segment are
// where the causal convolutions read their cached frames, so every conv is a plain GEMM over row-shifted taps.
// Kernel sequence: embedding gather, embed GEMM + LayerNorm (x sqrt(C) folded into its affine), the pre-lookahead conv1
// GEMM (4 taps, leaky ReLU epilogue), conv2's cache rows, conv2 GEMM (3 taps) + residual; per conformer layer: LN, QKV
// GEMM ([q + u | q + v | k | v]: the position biases folded into the bias), new keys into the pool, relative-position
// attention, output GEMM + residual, LN, w_1 GEMM (SiLU), w_2 GEMM + residual; the upsampling (nearest x2 with the
// cached frames) and its 5-tap conv GEMM, the up embed GEMM + LayerNorm, the second stack, after_norm, encoder_proj
// and the gather of each window's mu rows.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "cache_registry.h"
#include "common.cuh"
#include "enc_kernels.h"
#include "kernels.h"

using namespace t2w;

namespace {

#define E_CUDA(call)                     \
  do {                                   \
    cudaError_t e_ = (call);             \
    if (e_ != cudaSuccess) {             \
      set_cuda_error(e_);                \
      return T2W_ERR_CUDA;               \
    }                                    \
  } while (0)
#define E_TRY(call)         \
  do {                      \
    int rc_ = (call);       \
    if (rc_) return rc_;    \
  } while (0)

constexpr int kCacheFrames = 6;  // per stream: 2 frames of the pre-lookahead conv2's input, 4 of the upsampling conv's
constexpr int kMel = 80;

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct EncLayer {
  __nv_bfloat16 *w_qkv = nullptr, *w_out = nullptr, *w_ff1 = nullptr, *w_ff2 = nullptr, *pos = nullptr, *pool = nullptr;
  float *b_qkv = nullptr, *b_out = nullptr, *b_ff1 = nullptr, *b_ff2 = nullptr;
  float *nm_w = nullptr, *nm_b = nullptr, *nf_w = nullptr, *nf_b = nullptr;
  WeightMaps tm_qkv, tm_out, tm_ff1, tm_ff2;
};

// A stream's caches: first- and second-stack key slots in sequence order, its conv-cache row, the trim length.
struct EncRecord {
  bool live = false;
  uint32_t generation = 0;
  int32_t keep = 0, row = -1;
  std::vector<int32_t> k1, k2;
};

constexpr int kIndexBits = 20;
constexpr uint32_t kIndexMask = (1u << kIndexBits) - 1;

// The call's plan: row layout, index arrays (uploaded together) and the new slots of every window.
struct EncPlan {
  int n = 0, M1 = 0, M2 = 0, Mx = 0, n_out = 0;
  std::vector<int32_t> tok1;
  std::vector<uint8_t> pad_e1, pad1, pad2;
  std::vector<EncRow> er;
  std::vector<int32_t> sc1_row, sc1_slot, sc2_row, sc2_slot, kv1, kv2, out_src;
  std::vector<RelWork> w1, w2;
};

struct EncLayout {
  size_t tok1, pad_e1, pad1, pad2, er, sc1_row, sc1_slot, sc2_row, sc2_slot, kv1, kv2, w1, w2, out_src, meta_bytes;
  size_t h1, h2, a, qkv, o, f, y3, total;
};

}  // namespace

struct t2w_encoder {
  t2w_enc_config cfg{};
  int device = 0, max_frames = 0, n_slots1 = 0, n_slots2 = 0, n_streams = 0;
  std::vector<void*> allocs;
  __nv_bfloat16 *emb = nullptr, *w_embed = nullptr, *w_c1 = nullptr, *w_c2 = nullptr, *w_up = nullptr,
                *w_upemb = nullptr, *w_proj = nullptr, *cnn = nullptr;
  // K/V pools of the two stacks: [layers of the stack][slots][2 H], layer l's pool at l * slots * 2 H
  __nv_bfloat16 *pool1 = nullptr, *pool2 = nullptr;
  float *b_embed = nullptr, *b_c1 = nullptr, *b_c2 = nullptr, *b_up = nullptr, *b_upemb = nullptr, *b_proj = nullptr;
  float *ln_e_w = nullptr, *ln_e_b = nullptr, *ln_u_w = nullptr, *ln_u_b = nullptr, *ln_a_w = nullptr,
        *ln_a_b = nullptr, *ones = nullptr;
  WeightMaps tm_embed, tm_c1, tm_c2, tm_up, tm_upemb, tm_proj;
  std::vector<EncLayer> L;
  int* err = nullptr;
  SlotBitmap s1, s2, rows;
  std::vector<EncRecord> recs;
  std::vector<uint32_t> vacant;
  std::mutex mu;
  static constexpr int kStaging = 4;
  struct Staging {
    void* host = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;
    bool used = false;
  };
  Staging staging[kStaging];
  int staging_next = 0;
  // CUDA graphs of whole calls, per launch structure (sizes and buffers), captured the second time a key is seen
  struct CachedGraph {
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t done = nullptr;  // recorded after its latest launch: an evicted graph may still run on another stream
  };
  std::unordered_map<uint64_t, CachedGraph> graphs;
  std::unordered_map<uint64_t, int> seen;
  cudaStream_t cap_stream = nullptr;
  int64_t n_replays = 0, n_captures = 0, n_eager = 0;

  EncRecord* find(int32_t handle) {
    if (handle < 0) return nullptr;
    const uint32_t idx = (uint32_t)handle & kIndexMask, gen = (uint32_t)handle >> kIndexBits;
    if (idx >= recs.size()) return nullptr;
    EncRecord& r = recs[idx];
    return (r.live && r.generation == gen) ? &r : nullptr;
  }
  const EncRecord* find(int32_t handle) const { return const_cast<t2w_encoder*>(this)->find(handle); }
};

namespace {

// Makes the encoder's device current for a call and restores the caller's device afterwards.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) return;
    ok = prev == dev || cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

template <class T>
int dalloc(t2w_encoder* e, T** p, size_t n) {
  void* q = nullptr;
  const cudaError_t rc = cudaMalloc(&q, n * sizeof(T) > 0 ? n * sizeof(T) : 16);
  if (rc != cudaSuccess) {
    set_cuda_error(rc);
    return rc == cudaErrorMemoryAllocation ? T2W_ERR_OOM : T2W_ERR_CUDA;
  }
  e->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return T2W_OK;
}

int to_bf16(t2w_encoder* e, const float* src, size_t n, __nv_bfloat16** dst, cudaStream_t st) {
  E_TRY(dalloc(e, dst, n));
  return launch_f32_to_bf16(src, *dst, (long long)n, st);
}
int conv_w(t2w_encoder* e, const float* src, int C, int k, __nv_bfloat16** dst, cudaStream_t st) {
  E_TRY(dalloc(e, dst, (size_t)C * C * k));
  return launch_conv_weight(src, *dst, C, C, k, st);
}
int copy_f32(t2w_encoder* e, const float* src, size_t n, float** dst) {
  E_TRY(dalloc(e, dst, n));
  E_CUDA(cudaMemcpy(*dst, src, n * 4, cudaMemcpyDeviceToDevice));
  return T2W_OK;
}
int host_f32(const float* src, size_t n, std::vector<float>& out) {
  out.resize(n);
  E_CUDA(cudaMemcpy(out.data(), src, n * 4, cudaMemcpyDeviceToHost));
  return T2W_OK;
}
int upload_f32(t2w_encoder* e, const std::vector<float>& v, float** dst) {
  E_TRY(dalloc(e, dst, v.size()));
  E_CUDA(cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return T2W_OK;
}
// LayerNorm affine scaled by s (the embeddings' x sqrt(C) after their LayerNorm folds into it).
int scaled_ln(t2w_encoder* e, const float* w, const float* b, int C, float s, float** dw, float** db) {
  std::vector<float> hw, hb;
  E_TRY(host_f32(w, C, hw));
  E_TRY(host_f32(b, C, hb));
  for (int i = 0; i < C; ++i) {
    hw[i] *= s;
    hb[i] *= s;
  }
  E_TRY(upload_f32(e, hw, dw));
  return upload_f32(e, hb, db);
}

bool valid_cfg(const t2w_enc_config& c) {
  return c.vocab > 0 && c.head_dim == 64 && c.heads > 0 && c.hidden == 64 * c.heads && c.hidden % 128 == 0 &&
         c.hidden <= 1024 && c.ffn > 0 && c.ffn % 128 == 0 && c.blocks1 > 0 && c.blocks2 > 0 && c.stride == 2 &&
         c.lookahead == 3 && c.mel == kMel && c.eps_layer > 0 && c.eps_embed > 0 && c.eps_after > 0 &&
         c.max_period > 1.f;
}

int create_impl(t2w_encoder* e, const float* const* W, cudaStream_t st) {
  const t2w_enc_config& c = e->cfg;
  const int H = c.hidden, F = c.ffn, V = c.vocab;
  E_TRY(to_bf16(e, W[T2W_E_EMB], (size_t)V * H, &e->emb, st));
  E_TRY(to_bf16(e, W[T2W_E_EMBED_W], (size_t)H * H, &e->w_embed, st));
  E_TRY(copy_f32(e, W[T2W_E_EMBED_B], H, &e->b_embed));
  E_TRY(scaled_ln(e, W[T2W_E_EMBED_LN_W], W[T2W_E_EMBED_LN_B], H, std::sqrt((float)H), &e->ln_e_w, &e->ln_e_b));
  E_TRY(conv_w(e, W[T2W_E_PL_C1_W], H, c.lookahead + 1, &e->w_c1, st));
  E_TRY(copy_f32(e, W[T2W_E_PL_C1_B], H, &e->b_c1));
  E_TRY(conv_w(e, W[T2W_E_PL_C2_W], H, 3, &e->w_c2, st));
  E_TRY(copy_f32(e, W[T2W_E_PL_C2_B], H, &e->b_c2));
  E_TRY(conv_w(e, W[T2W_E_UP_W], H, 2 * c.stride + 1, &e->w_up, st));
  E_TRY(copy_f32(e, W[T2W_E_UP_B], H, &e->b_up));
  E_TRY(to_bf16(e, W[T2W_E_UPEMB_W], (size_t)H * H, &e->w_upemb, st));
  E_TRY(copy_f32(e, W[T2W_E_UPEMB_B], H, &e->b_upemb));
  E_TRY(scaled_ln(e, W[T2W_E_UPEMB_LN_W], W[T2W_E_UPEMB_LN_B], H, std::sqrt((float)H), &e->ln_u_w, &e->ln_u_b));
  E_TRY(copy_f32(e, W[T2W_E_AFTER_W], H, &e->ln_a_w));
  E_TRY(copy_f32(e, W[T2W_E_AFTER_B], H, &e->ln_a_b));
  E_TRY(to_bf16(e, W[T2W_E_PROJ_W], (size_t)kMel * H, &e->w_proj, st));
  E_TRY(copy_f32(e, W[T2W_E_PROJ_B], kMel, &e->b_proj));
  E_TRY(upload_f32(e, std::vector<float>(H, 1.f), &e->ones));
  if (!make_weight_maps(&e->tm_embed, e->w_embed, H, H) || !make_weight_maps(&e->tm_c1, e->w_c1, H, 4 * H) ||
      !make_weight_maps(&e->tm_c2, e->w_c2, H, 3 * H) || !make_weight_maps(&e->tm_up, e->w_up, H, 5 * H) ||
      !make_weight_maps(&e->tm_upemb, e->w_upemb, H, H) || !make_weight_maps(&e->tm_proj, e->w_proj, kMel, H))
    return T2W_ERR_INVALID;
  const int nl = c.blocks1 + c.blocks2;
  e->L.resize(nl);
  E_TRY(dalloc(e, &e->pool1, (size_t)c.blocks1 * e->n_slots1 * 2 * H));
  E_TRY(dalloc(e, &e->pool2, (size_t)c.blocks2 * e->n_slots2 * 2 * H));
  const size_t rows_pos = (size_t)(2 * e->max_frames - 1);
  for (int l = 0; l < nl; ++l) {
    const float* const* lw = W + T2W_E_COUNT + (size_t)l * T2W_EL_COUNT;
    EncLayer& y = e->L[l];
    // [q + u | q + v | k | v]: linear_q twice, its bias plus pos_bias_u / pos_bias_v
    E_TRY(dalloc(e, &y.w_qkv, (size_t)4 * H * H));
    const float* blocks[4] = {lw[T2W_EL_Q_W], lw[T2W_EL_Q_W], lw[T2W_EL_K_W], lw[T2W_EL_V_W]};
    for (int q = 0; q < 4; ++q) E_TRY(launch_f32_to_bf16(blocks[q], y.w_qkv + (size_t)q * H * H, (long long)H * H, st));
    std::vector<float> bq, bk, bv, pu, pv;
    E_TRY(host_f32(lw[T2W_EL_Q_B], H, bq));
    E_TRY(host_f32(lw[T2W_EL_K_B], H, bk));
    E_TRY(host_f32(lw[T2W_EL_V_B], H, bv));
    E_TRY(host_f32(lw[T2W_EL_POS_U], H, pu));
    E_TRY(host_f32(lw[T2W_EL_POS_V], H, pv));
    std::vector<float> b4((size_t)4 * H);
    for (int i = 0; i < H; ++i) {
      b4[i] = bq[i] + pu[i];
      b4[H + i] = bq[i] + pv[i];
      b4[2 * H + i] = bk[i];
      b4[3 * H + i] = bv[i];
    }
    E_TRY(upload_f32(e, b4, &y.b_qkv));
    E_TRY(to_bf16(e, lw[T2W_EL_OUT_W], (size_t)H * H, &y.w_out, st));
    E_TRY(copy_f32(e, lw[T2W_EL_OUT_B], H, &y.b_out));
    E_TRY(to_bf16(e, lw[T2W_EL_FF1_W], (size_t)F * H, &y.w_ff1, st));
    E_TRY(copy_f32(e, lw[T2W_EL_FF1_B], F, &y.b_ff1));
    E_TRY(to_bf16(e, lw[T2W_EL_FF2_W], (size_t)H * F, &y.w_ff2, st));
    E_TRY(copy_f32(e, lw[T2W_EL_FF2_B], H, &y.b_ff2));
    E_TRY(copy_f32(e, lw[T2W_EL_NMHA_W], H, &y.nm_w));
    E_TRY(copy_f32(e, lw[T2W_EL_NMHA_B], H, &y.nm_b));
    E_TRY(copy_f32(e, lw[T2W_EL_NFF_W], H, &y.nf_w));
    E_TRY(copy_f32(e, lw[T2W_EL_NFF_B], H, &y.nf_b));
    E_TRY(dalloc(e, &y.pos, rows_pos * H));
    E_TRY(launch_pos_table(lw[T2W_EL_POS_W], H, e->max_frames, c.max_period, y.pos, st));
    y.pool = l < c.blocks1 ? e->pool1 + (size_t)l * e->n_slots1 * 2 * H
                           : e->pool2 + (size_t)(l - c.blocks1) * e->n_slots2 * 2 * H;
    if (!make_weight_maps(&y.tm_qkv, y.w_qkv, 4 * H, H) || !make_weight_maps(&y.tm_out, y.w_out, H, H) ||
        !make_weight_maps(&y.tm_ff1, y.w_ff1, F, H) || !make_weight_maps(&y.tm_ff2, y.w_ff2, H, F))
      return T2W_ERR_INVALID;
  }
  E_TRY(dalloc(e, &e->cnn, (size_t)e->n_streams * kCacheFrames * H));
  E_CUDA(cudaMemsetAsync(e->cnn, 0, (size_t)e->n_streams * kCacheFrames * H * 2, st));
  E_TRY(dalloc(e, &e->err, 1));
  E_CUDA(cudaMemsetAsync(e->err, 0, 4, st));
  e->s1.init(e->n_slots1, 0);
  e->s2.init(e->n_slots2, 0);
  e->rows.init(e->n_streams, 0);
  E_CUDA(cudaStreamSynchronize(st));
  return T2W_OK;
}

void free_all(t2w_encoder* e) {
  for (auto& kv : e->graphs) {
    if (kv.second.done) cudaEventSynchronize(kv.second.done);
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.done) cudaEventDestroy(kv.second.done);
  }
  e->graphs.clear();
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  e->cap_stream = nullptr;
  for (void* p : e->allocs) cudaFree(p);
  e->allocs.clear();
  for (auto& sg : e->staging) {
    if (sg.done) cudaEventDestroy(sg.done);
    if (sg.host) cudaFreeHost(sg.host);
    sg = t2w_encoder::Staging();
  }
}

// Frames of a window: its tokens minus the look-ahead ones, or all of them for a final window.
int frames_of(const t2w_enc_config& c, int n_tok, bool fin) { return fin ? n_tok : n_tok - c.lookahead; }

// Validates the batch against the records (under the lock) and fills the plan's sizes and index arrays; new slots
// are taken only when `take` is set (the workspace query plans without them).
int plan_call(t2w_encoder* e, const t2w_enc_batch& b, bool take, EncPlan& pl) {
  const t2w_enc_config& c = e->cfg;
  const int n = b.n_streams;
  if (n <= 0 || !b.handle || !b.n_tokens || !b.final || !b.tokens) return T2W_ERR_INVALID;
  pl = EncPlan();
  pl.n = n;
  std::vector<EncRecord*> rec(n);
  long long rows1 = 0, rows2 = 0, new1 = 0, new2 = 0, ntok = 0, nkv1 = 0, nkv2 = 0;
  for (int i = 0; i < n; ++i) {
    rec[i] = e->find(b.handle[i]);
    if (!rec[i]) return T2W_ERR_INVALID;
    for (int j = 0; j < i; ++j)
      if (b.handle[j] == b.handle[i]) return T2W_ERR_INVALID;
    const bool fin = b.final[i] != 0;
    const int T = frames_of(c, b.n_tokens[i], fin);
    if (b.n_tokens[i] <= 0 || T < 1 || (!fin && T < 2)) return T2W_ERR_INVALID;
    const long long K1 = (long long)rec[i]->k1.size() + T, K2 = (long long)rec[i]->k2.size() + 2ll * T;
    if (2ll * T > e->max_frames || K1 > e->max_frames || K2 > e->max_frames) return T2W_ERR_INVALID;
    rows1 += T + 5;
    rows2 += 2ll * T + 4;
    new1 += T;
    new2 += 2ll * T;
    nkv1 += K1;
    nkv2 += K2;
    ntok += b.n_tokens[i];
  }
  if (rows2 > (1ll << 30) || ntok > (1ll << 30)) return T2W_ERR_INVALID;
  for (long long t = 0; t < ntok; ++t)
    if (b.tokens[t] < 0 || b.tokens[t] >= c.vocab) return T2W_ERR_INVALID;
  if (new1 > e->s1.available() || new2 > e->s2.available()) return T2W_ERR_EXHAUSTED;
  pl.M1 = (int)((rows1 + 127) / 128 * 128);
  pl.M2 = (int)((rows2 + 127) / 128 * 128);
  pl.Mx = std::max(pl.M1, pl.M2);
  pl.n_out = (int)new2;
  if (!take) {  // sizes only: the index arrays' lengths
    pl.tok1.resize(pl.M1);
    pl.pad_e1.resize(pl.M1);
    pl.pad1.resize(pl.M1);
    pl.pad2.resize(pl.M2);
    pl.er.resize(n);
    pl.sc1_row.resize(new1);
    pl.sc1_slot.resize(new1);
    pl.sc2_row.resize(new2);
    pl.sc2_slot.resize(new2);
    pl.kv1.resize(nkv1);
    pl.kv2.resize(nkv2);
    long long nw1 = 0, nw2 = 0;
    for (int i = 0; i < n; ++i) {
      const int T = frames_of(c, b.n_tokens[i], b.final[i] != 0);
      nw1 += (T + 127) / 128;
      nw2 += (2 * T + 127) / 128;
    }
    pl.w1.resize(nw1);
    pl.w2.resize(nw2);
    pl.out_src.resize(new2);
    return T2W_OK;
  }
  pl.tok1.assign(pl.M1, -1);
  pl.pad_e1.assign(pl.M1, 1);
  pl.pad1.assign(pl.M1, 1);
  pl.pad2.assign(pl.M2, 1);
  pl.er.resize(n);
  int seg1 = 0, seg2 = 0;
  long long tk = 0;
  std::vector<int32_t> fresh1((size_t)new1), fresh2((size_t)new2);
  if (!e->s1.take((int)new1, fresh1.data())) return T2W_ERR_EXHAUSTED;
  if (!e->s2.take((int)new2, fresh2.data())) {
    e->s1.give(fresh1.data(), fresh1.size());
    return T2W_ERR_EXHAUSTED;
  }
  size_t f1 = 0, f2 = 0;
  for (int i = 0; i < n; ++i) {
    const bool fin = b.final[i] != 0;
    const int nt = b.n_tokens[i], T = frames_of(c, nt, fin);
    EncRecord& r = *rec[i];
    pl.er[i] = EncRow{seg1, T, r.row, seg2};
    for (int t = 0; t < nt; ++t) pl.tok1[seg1 + 2 + t] = b.tokens[tk + t];
    tk += nt;
    for (int t = 0; t < T + (fin ? 0 : c.lookahead); ++t) pl.pad_e1[seg1 + 2 + t] = 0;
    for (int t = 0; t < T; ++t) pl.pad1[seg1 + 2 + t] = 0;
    for (int t = 0; t < 2 * T; ++t) pl.pad2[seg2 + 4 + t] = 0;
    // stack 1: keys [cached | new], queries the window's frames
    const int kv1_off = (int)pl.kv1.size(), K1 = (int)r.k1.size() + T;
    pl.kv1.insert(pl.kv1.end(), r.k1.begin(), r.k1.end());
    for (int t = 0; t < T; ++t) {
      const int32_t sl = fresh1[f1++];
      pl.kv1.push_back(sl);
      pl.sc1_row.push_back(seg1 + 2 + t);
      pl.sc1_slot.push_back(sl);
    }
    for (int q = 0; q < T; q += 128) pl.w1.push_back(RelWork{seg1 + 2 + q, q, T, K1, kv1_off});
    const int kv2_off = (int)pl.kv2.size(), K2 = (int)r.k2.size() + 2 * T;
    pl.kv2.insert(pl.kv2.end(), r.k2.begin(), r.k2.end());
    for (int t = 0; t < 2 * T; ++t) {
      const int32_t sl = fresh2[f2++];
      pl.kv2.push_back(sl);
      pl.sc2_row.push_back(seg2 + 4 + t);
      pl.sc2_slot.push_back(sl);
      pl.out_src.push_back(seg2 + 4 + t);
    }
    for (int q = 0; q < 2 * T; q += 128) pl.w2.push_back(RelWork{seg2 + 4 + q, q, 2 * T, K2, kv2_off});
    seg1 += T + 5;
    seg2 += 2 * T + 4;
  }
  return T2W_OK;
}

EncLayout layout_of(const t2w_enc_config& c, const EncPlan& pl) {
  EncLayout L{};
  size_t o = 0;
  auto put = [&](size_t& f, size_t bytes) {
    f = o;
    o = a256(o + bytes);
  };
  put(L.tok1, pl.tok1.size() * 4);
  put(L.pad_e1, pl.pad_e1.size());
  put(L.pad1, pl.pad1.size());
  put(L.pad2, pl.pad2.size());
  put(L.er, pl.er.size() * sizeof(EncRow));
  put(L.sc1_row, pl.sc1_row.size() * 4);
  put(L.sc1_slot, pl.sc1_slot.size() * 4);
  put(L.sc2_row, pl.sc2_row.size() * 4);
  put(L.sc2_slot, pl.sc2_slot.size() * 4);
  put(L.kv1, pl.kv1.size() * 4);
  put(L.kv2, pl.kv2.size() * 4);
  put(L.w1, pl.w1.size() * sizeof(RelWork));
  put(L.w2, pl.w2.size() * sizeof(RelWork));
  put(L.out_src, pl.out_src.size() * 4);
  L.meta_bytes = o;
  const size_t H = c.hidden, F = c.ffn;
  put(L.h1, (size_t)pl.M1 * H * 4);
  put(L.h2, (size_t)pl.M2 * H * 4);
  put(L.a, (size_t)pl.Mx * H * 2);
  put(L.qkv, (size_t)pl.Mx * 4 * H * 2);
  put(L.o, (size_t)pl.Mx * H * 2);
  put(L.f, (size_t)pl.Mx * F * 2);
  put(L.y3, (size_t)pl.M2 * kMel * 4);
  L.total = o;
  return L;
}

template <class T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off);
}

int upload(t2w_encoder* e, const EncPlan& pl, const EncLayout& L, void* ws, cudaStream_t st) {
  t2w_encoder::Staging& sg = e->staging[e->staging_next];
  e->staging_next = (e->staging_next + 1) % t2w_encoder::kStaging;
  if (sg.used) E_CUDA(cudaEventSynchronize(sg.done));
  if (sg.cap < L.meta_bytes) {
    if (sg.host) cudaFreeHost(sg.host);
    sg.host = nullptr;
    sg.cap = 0;
    const size_t cap = std::max<size_t>(L.meta_bytes + L.meta_bytes / 4, 1 << 16);
    E_CUDA(cudaMallocHost(&sg.host, cap));
    sg.cap = cap;
  }
  if (!sg.done) E_CUDA(cudaEventCreateWithFlags(&sg.done, cudaEventDisableTiming));
  uint8_t* img = static_cast<uint8_t*>(sg.host);
  auto put = [&](size_t off, const void* src, size_t bytes) {
    if (bytes) std::memcpy(img + off, src, bytes);
  };
  put(L.tok1, pl.tok1.data(), pl.tok1.size() * 4);
  put(L.pad_e1, pl.pad_e1.data(), pl.pad_e1.size());
  put(L.pad1, pl.pad1.data(), pl.pad1.size());
  put(L.pad2, pl.pad2.data(), pl.pad2.size());
  put(L.er, pl.er.data(), pl.er.size() * sizeof(EncRow));
  put(L.sc1_row, pl.sc1_row.data(), pl.sc1_row.size() * 4);
  put(L.sc1_slot, pl.sc1_slot.data(), pl.sc1_slot.size() * 4);
  put(L.sc2_row, pl.sc2_row.data(), pl.sc2_row.size() * 4);
  put(L.sc2_slot, pl.sc2_slot.data(), pl.sc2_slot.size() * 4);
  put(L.kv1, pl.kv1.data(), pl.kv1.size() * 4);
  put(L.kv2, pl.kv2.data(), pl.kv2.size() * 4);
  put(L.w1, pl.w1.data(), pl.w1.size() * sizeof(RelWork));
  put(L.w2, pl.w2.data(), pl.w2.size() * sizeof(RelWork));
  put(L.out_src, pl.out_src.data(), pl.out_src.size() * 4);
  E_CUDA(cudaMemcpyAsync(ws, img, L.meta_bytes, cudaMemcpyHostToDevice, st));
  E_CUDA(cudaEventRecord(sg.done, st));
  sg.used = true;
  return T2W_OK;
}

int gemm(const void* A, int rows_a, const void* Wt, const WeightMaps* wm, const float* bias, int M, int N, int K,
         int taps, int tap_row0, int epi, void* out, int ldo, const float* gate, float slope, int* err, cudaStream_t st) {
  GemmArgs g;
  g.A = A;
  g.lda = K;
  g.rows_a = rows_a;
  g.W = Wt;
  g.bias = bias;
  g.M = M;
  g.N = N;
  g.K = K;
  g.taps = taps;
  g.tap_row0 = tap_row0;
  g.epi = epi;
  g.out = out;
  g.ldo = ldo;
  g.gate = gate;
  g.qk_eps = slope;
  g.err = err;
  return launch_gemm(g, st, nullptr, wm);
}

// One conformer layer over the rows of h (fp32 residual stream of M rows; pad marks rows that are not frames).
int run_layer(t2w_encoder* e, const EncLayer& y, float* h, int M, const uint8_t* pad, const int* sc_row,
              const int* sc_slot, int n_sc, const RelWork* work, int n_work, const int* kv_idx, void* ws,
              const EncLayout& Lo, const EncPlan& pl, cudaStream_t st) {
  const t2w_enc_config& c = e->cfg;
  const int H = c.hidden, F = c.ffn;
  __nv_bfloat16* a = at<__nv_bfloat16>(ws, Lo.a);
  __nv_bfloat16* qkv = at<__nv_bfloat16>(ws, Lo.qkv);
  __nv_bfloat16* o = at<__nv_bfloat16>(ws, Lo.o);
  __nv_bfloat16* f = at<__nv_bfloat16>(ws, Lo.f);
  E_TRY(launch_enc_ln(h, y.nm_w, y.nm_b, c.eps_layer, M, H, nullptr, a, pad, st));
  E_TRY(gemm(a, M, y.w_qkv, &y.tm_qkv, y.b_qkv, M, 4 * H, H, 1, 0, T2W_EPI_BF16, qkv, 4 * H, nullptr, 0.f, e->err, st));
  E_TRY(launch_enc_kv_scatter(qkv, H, sc_row, sc_slot, n_sc, y.pool, st));
  CUtensorMap tq, tp;
  if (!make_relattn_tmaps(&tq, &tp, qkv, pl.Mx, H, y.pos, e->max_frames)) return T2W_ERR_INVALID;
  RelArgs ra;
  ra.work = work;
  ra.n_work = n_work;
  ra.heads = c.heads;
  ra.pool = y.pool;
  ra.pool_ld = 2 * H;
  ra.kv_idx = kv_idx;
  ra.r0 = e->max_frames - 1;
  ra.out = o;
  ra.ldo = H;
  ra.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)c.head_dim));
  ra.err = e->err;
  E_TRY(launch_relattn(ra, tq, tp, st));
  E_TRY(gemm(o, M, y.w_out, &y.tm_out, y.b_out, M, H, H, 1, 0, T2W_EPI_RESID, h, H, e->ones, 0.f, e->err, st));
  E_TRY(launch_enc_ln(h, y.nf_w, y.nf_b, c.eps_layer, M, H, nullptr, a, pad, st));
  E_TRY(gemm(a, M, y.w_ff1, &y.tm_ff1, y.b_ff1, M, F, H, 1, 0, T2W_EPI_SILU, f, F, nullptr, 0.f, e->err, st));
  return gemm(f, M, y.w_ff2, &y.tm_ff2, y.b_ff2, M, H, F, 1, 0, T2W_EPI_RESID, h, H, e->ones, 0.f, e->err, st);
}

int run_call(t2w_encoder* e, const EncPlan& pl, const EncLayout& Lo, void* ws, float* mu, cudaStream_t st) {
  const t2w_enc_config& c = e->cfg;
  const int H = c.hidden;
  float* h1 = at<float>(ws, Lo.h1);
  float* h2 = at<float>(ws, Lo.h2);
  __nv_bfloat16* a = at<__nv_bfloat16>(ws, Lo.a);
  __nv_bfloat16* o = at<__nv_bfloat16>(ws, Lo.o);
  float* y3 = at<float>(ws, Lo.y3);
  const EncRow* er = at<EncRow>(ws, Lo.er);
  // stack 1: embedding, embed linear + LayerNorm (x sqrt(C)), pre-lookahead layer
  E_TRY(launch_embed_rows(e->emb, at<int>(ws, Lo.tok1), pl.M1, H, o, st));
  E_TRY(gemm(o, pl.M1, e->w_embed, &e->tm_embed, e->b_embed, pl.M1, H, H, 1, 0, T2W_EPI_F32, h1, H, nullptr, 0.f,
             e->err, st));
  E_TRY(launch_enc_ln(h1, e->ln_e_w, e->ln_e_b, c.eps_embed, pl.M1, H, h1, a, at<uint8_t>(ws, Lo.pad_e1), st));
  E_TRY(gemm(a, pl.M1, e->w_c1, &e->tm_c1, e->b_c1, pl.M1, H, H, c.lookahead + 1, 0, T2W_EPI_LEAKY, o, H, nullptr,
             c.leaky_slope, e->err, st));
  E_TRY(launch_pl_cache(o, H, er, pl.n, e->cnn, kCacheFrames, st));
  E_TRY(gemm(o, pl.M1, e->w_c2, &e->tm_c2, e->b_c2, pl.M1, H, H, 3, -2, T2W_EPI_RESID, h1, H, e->ones, 0.f, e->err, st));
  for (int l = 0; l < c.blocks1; ++l)
    E_TRY(run_layer(e, e->L[l], h1, pl.M1, at<uint8_t>(ws, Lo.pad1), at<int>(ws, Lo.sc1_row), at<int>(ws, Lo.sc1_slot),
                    (int)pl.sc1_row.size(), at<RelWork>(ws, Lo.w1), (int)pl.w1.size(), at<int>(ws, Lo.kv1), ws, Lo, pl,
                    st));
  // upsampling: nearest x2 after the cached frames, the 5-tap conv, up embed linear + LayerNorm (x sqrt(C))
  E_TRY(launch_up_pack(h1, H, er, pl.n, o, e->cnn, kCacheFrames, st));
  E_TRY(gemm(o, pl.M2, e->w_up, &e->tm_up, e->b_up, pl.M2, H, H, 2 * c.stride + 1, -2 * c.stride, T2W_EPI_BF16, a, H,
             nullptr, 0.f, e->err, st));
  E_TRY(gemm(a, pl.M2, e->w_upemb, &e->tm_upemb, e->b_upemb, pl.M2, H, H, 1, 0, T2W_EPI_F32, h2, H, nullptr, 0.f,
             e->err, st));
  E_TRY(launch_enc_ln(h2, e->ln_u_w, e->ln_u_b, c.eps_embed, pl.M2, H, h2, nullptr, at<uint8_t>(ws, Lo.pad2), st));
  for (int l = 0; l < c.blocks2; ++l)
    E_TRY(run_layer(e, e->L[c.blocks1 + l], h2, pl.M2, at<uint8_t>(ws, Lo.pad2), at<int>(ws, Lo.sc2_row),
                    at<int>(ws, Lo.sc2_slot), (int)pl.sc2_row.size(), at<RelWork>(ws, Lo.w2), (int)pl.w2.size(),
                    at<int>(ws, Lo.kv2), ws, Lo, pl, st));
  E_TRY(launch_enc_ln(h2, e->ln_a_w, e->ln_a_b, c.eps_after, pl.M2, H, nullptr, a, at<uint8_t>(ws, Lo.pad2), st));
  E_TRY(gemm(a, pl.M2, e->w_proj, &e->tm_proj, e->b_proj, pl.M2, kMel, H, 1, 0, T2W_EPI_F32, y3, kMel, nullptr, 0.f,
             e->err, st));
  return launch_gather_rows_f32(y3, kMel, at<int>(ws, Lo.out_src), pl.n_out, mu, st);
}

uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h * 0xff51afd7ed558ccdull;
}

// The launches of a call depend only on the plan's sizes and the buffers (the index arrays are read from the
// workspace, where upload() has just put this call's): one graph per such key.
uint64_t call_key(const EncPlan& pl, const void* ws, const void* mu) {
  uint64_t k = 0xE0C0DE5ull;
  for (long long v : {(long long)pl.n, (long long)pl.M1, (long long)pl.M2, (long long)pl.n_out,
                      (long long)pl.sc1_row.size(), (long long)pl.sc2_row.size(), (long long)pl.kv1.size(),
                      (long long)pl.kv2.size(), (long long)pl.w1.size(), (long long)pl.w2.size()})
    k = mix(k, (uint64_t)v);
  return mix(mix(k, reinterpret_cast<uint64_t>(ws)), reinterpret_cast<uint64_t>(mu));
}

constexpr size_t kMaxGraphs = 64;

template <class F>
int replay(t2w_encoder* e, uint64_t key, cudaStream_t st, F&& enqueue) {
  auto g = e->graphs.find(key);
  if (g == e->graphs.end()) {
    cudaStreamCaptureStatus cs;
    E_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;  // the caller is capturing: use flags = 0
    if (e->graphs.size() >= kMaxGraphs) {  // drop one, once its latest launch (on whichever stream) has finished
      auto victim = e->graphs.begin();
      E_CUDA(cudaEventSynchronize(victim->second.done));
      cudaGraphExecDestroy(victim->second.exec);
      cudaEventDestroy(victim->second.done);
      e->graphs.erase(victim);
    }
    if (!e->cap_stream) E_CUDA(cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking));
    E_CUDA(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue(e->cap_stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(e->cap_stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ec != cudaSuccess) {
      set_cuda_error(ec);
      return T2W_ERR_CUDA;
    }
    t2w_encoder::CachedGraph cg;
    const cudaError_t ei = cudaGraphInstantiate(&cg.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) {
      set_cuda_error(ei);
      return T2W_ERR_CUDA;
    }
    const cudaError_t ee = cudaEventCreateWithFlags(&cg.done, cudaEventDisableTiming);
    if (ee != cudaSuccess) {
      cudaGraphExecDestroy(cg.exec);
      set_cuda_error(ee);
      return T2W_ERR_CUDA;
    }
    g = e->graphs.emplace(key, cg).first;
    ++e->n_captures;
  }
  E_CUDA(cudaGraphLaunch(g->second.exec, st));
  E_CUDA(cudaEventRecord(g->second.done, st));
  ++e->n_replays;
  return T2W_OK;
}

// The caches after a window (token2wav_batch.py:395 trims conformer_att_cache along time to its first keep and last
// 100 frames; the first stack's cache is stored tiled twice and read back as the first half of the cut).
void advance(t2w_encoder* e, EncRecord& r, const int32_t* new1, int T) {
  const long long keep = r.keep < 0 ? 0 : r.keep;
  // first stack: [cached | new]; tiled length 2 K1 cut to keep + 100, whose first half is a prefix of the list
  r.k1.insert(r.k1.end(), new1, new1 + T);
  const long long K1 = (long long)r.k1.size();
  if (2 * K1 > keep + kTrimSuffix) {
    const size_t n1 = (size_t)((keep + kTrimSuffix) / 2);
    e->s1.give(r.k1.data() + n1, r.k1.size() - n1);
    r.k1.resize(n1);
  }
}
void advance2(t2w_encoder* e, EncRecord& r, const int32_t* new2, int T2) {
  const long long keep = r.keep < 0 ? 0 : r.keep;
  r.k2.insert(r.k2.end(), new2, new2 + T2);
  if ((long long)r.k2.size() > keep + kTrimSuffix) {
    const size_t c0 = (size_t)keep, c1 = r.k2.size() - kTrimSuffix;
    e->s2.give(r.k2.data() + c0, c1 - c0);
    r.k2.erase(r.k2.begin() + c0, r.k2.begin() + c1);
  }
}

}  // namespace

extern "C" {

int t2w_encoder_create(const t2w_enc_config* cfg, const float* const* weights, int32_t n_weights, int32_t max_frames,
                       int32_t n_slots1, int32_t n_slots2, int32_t n_streams, void* stream, t2w_encoder** out) {
  if (!cfg || !weights || !out || !valid_cfg(*cfg) || max_frames < 8 || max_frames > 65536 || n_slots1 <= 0 ||
      n_slots2 <= 0 || n_streams <= 0 || n_streams > (int)kIndexMask)
    return T2W_ERR_INVALID;
  const int nl = cfg->blocks1 + cfg->blocks2;
  if (n_weights != T2W_E_COUNT + nl * T2W_EL_COUNT) return T2W_ERR_INVALID;
  for (int i = 0; i < n_weights; ++i)
    if (!weights[i]) return T2W_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || !t2w_device_ok(dev)) return T2W_ERR_UNSUPPORTED;
  t2w_encoder* e = new t2w_encoder();
  e->cfg = *cfg;
  e->device = dev;
  e->max_frames = max_frames;
  e->n_slots1 = n_slots1;
  e->n_slots2 = n_slots2;
  e->n_streams = n_streams;
  const int rc = create_impl(e, weights, static_cast<cudaStream_t>(stream));
  if (rc) {
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    free_all(e);
    delete e;
    return rc;
  }
  *out = e;
  return T2W_OK;
}

int t2w_encoder_destroy(t2w_encoder* e) {
  if (!e) return T2W_ERR_INVALID;
  DeviceGuard g(e->device);
  cudaDeviceSynchronize();
  free_all(e);
  delete e;
  return T2W_OK;
}

int t2w_enc_stream_new(t2w_encoder* e, int32_t keep, void* stream, int32_t* handle) {
  if (!e || !handle || keep < 0) return T2W_ERR_INVALID;
  DeviceGuard g(e->device);
  if (!g.ok) return T2W_ERR_CUDA;
  std::lock_guard<std::mutex> lk(e->mu);
  int32_t row;
  if (!e->rows.take(1, &row)) return T2W_ERR_EXHAUSTED;
  uint32_t idx;
  if (!e->vacant.empty()) {
    idx = e->vacant.back();
    e->vacant.pop_back();
  } else {
    idx = (uint32_t)e->recs.size();
    e->recs.emplace_back();
  }
  EncRecord& r = e->recs[idx];
  r.live = true;
  r.generation = (r.generation + 1) & ((1u << (31 - kIndexBits)) - 1);
  r.keep = keep;
  r.row = row;
  r.k1.clear();
  r.k2.clear();
  const size_t fb = (size_t)kCacheFrames * e->cfg.hidden * 2;
  const cudaError_t rc = cudaMemsetAsync(reinterpret_cast<uint8_t*>(e->cnn) + (size_t)row * fb, 0, fb,
                                         static_cast<cudaStream_t>(stream));
  if (rc != cudaSuccess) {
    set_cuda_error(rc);
    r.live = false;
    e->vacant.push_back(idx);
    e->rows.give(&row, 1);
    return T2W_ERR_CUDA;
  }
  *handle = (int32_t)((r.generation << kIndexBits) | idx);
  return T2W_OK;
}

int t2w_enc_stream_clone(t2w_encoder* e, int32_t handle, void* stream, int32_t* out) {
  if (!e || !out) return T2W_ERR_INVALID;
  DeviceGuard g(e->device);
  if (!g.ok) return T2W_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lk(e->mu);
  EncRecord* src = e->find(handle);
  if (!src) return T2W_ERR_INVALID;
  const int n1 = (int)src->k1.size(), n2 = (int)src->k2.size();
  std::vector<int32_t> ids((size_t)2 * (n1 + n2));  // [src1 | dst1 | src2 | dst2]
  int32_t row;
  if (!e->rows.take(1, &row)) return T2W_ERR_EXHAUSTED;
  int32_t* dst1 = ids.data() + n1;
  int32_t* dst2 = ids.data() + 2 * n1 + n2;
  if (!e->s1.take(n1, dst1)) {
    e->rows.give(&row, 1);
    return T2W_ERR_EXHAUSTED;
  }
  if (!e->s2.take(n2, dst2)) {
    e->s1.give(dst1, n1);
    e->rows.give(&row, 1);
    return T2W_ERR_EXHAUSTED;
  }
  std::copy(src->k1.begin(), src->k1.end(), ids.begin());
  std::copy(src->k2.begin(), src->k2.end(), ids.begin() + 2 * n1);
  auto undo = [&](int rc) {
    e->s1.give(dst1, n1);
    e->s2.give(dst2, n2);
    e->rows.give(&row, 1);
    return rc;
  };
  const int H = e->cfg.hidden;
  if (!ids.empty()) {
    int* d = nullptr;
    cudaError_t ce = cudaMallocAsync(reinterpret_cast<void**>(&d), ids.size() * 4, st);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(d, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) {
      set_cuda_error(ce);
      return undo(T2W_ERR_CUDA);
    }
    int rc = launch_slot_copy(e->pool1, 2 * H, (long long)e->n_slots1 * 2 * H, e->cfg.blocks1, d, d + n1, n1, st);
    if (!rc)
      rc = launch_slot_copy(e->pool2, 2 * H, (long long)e->n_slots2 * 2 * H, e->cfg.blocks2, d + 2 * n1,
                            d + 2 * n1 + n2, n2, st);
    cudaFreeAsync(d, st);
    if (rc) {
      cudaStreamSynchronize(st);
      return undo(rc);
    }
  }
  const size_t fb = (size_t)kCacheFrames * H;
  const cudaError_t cc = cudaMemcpyAsync(e->cnn + (size_t)row * fb, e->cnn + (size_t)src->row * fb, fb * 2,
                                         cudaMemcpyDeviceToDevice, st);
  if (cc != cudaSuccess) {
    set_cuda_error(cc);
    cudaStreamSynchronize(st);
    return undo(T2W_ERR_CUDA);
  }
  uint32_t idx;
  if (!e->vacant.empty()) {
    idx = e->vacant.back();
    e->vacant.pop_back();
  } else {
    idx = (uint32_t)e->recs.size();
    e->recs.emplace_back();
    src = e->find(handle);  // the records may have moved
  }
  EncRecord& r = e->recs[idx];
  r.live = true;
  r.generation = (r.generation + 1) & ((1u << (31 - kIndexBits)) - 1);
  r.keep = src->keep;
  r.row = row;
  r.k1.assign(dst1, dst1 + n1);
  r.k2.assign(dst2, dst2 + n2);
  *out = (int32_t)((r.generation << kIndexBits) | idx);
  return T2W_OK;
}

int t2w_enc_stream_release(t2w_encoder* e, int32_t handle) {
  if (!e) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lk(e->mu);
  EncRecord* r = e->find(handle);
  if (!r) return T2W_ERR_INVALID;
  e->s1.give(r->k1.data(), r->k1.size());
  e->s2.give(r->k2.data(), r->k2.size());
  r->k1.clear();
  r->k2.clear();
  e->rows.give(&r->row, 1);
  r->row = -1;
  r->live = false;
  e->vacant.push_back((uint32_t)handle & kIndexMask);
  return T2W_OK;
}

int t2w_enc_stream_get(const t2w_encoder* e, int32_t handle, int32_t* keys1, int32_t* keys2, int32_t* keep) {
  if (!e) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lk(const_cast<t2w_encoder*>(e)->mu);
  const EncRecord* r = e->find(handle);
  if (!r) return T2W_ERR_INVALID;
  if (keys1) *keys1 = (int32_t)r->k1.size();
  if (keys2) *keys2 = (int32_t)r->k2.size();
  if (keep) *keep = r->keep;
  return T2W_OK;
}

int t2w_enc_usage(const t2w_encoder* e, int32_t* slots1, int32_t* slots2, int32_t* streams) {
  if (!e) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lk(const_cast<t2w_encoder*>(e)->mu);
  if (slots1) *slots1 = e->s1.used();
  if (slots2) *slots2 = e->s2.used();
  if (streams) *streams = e->rows.used();
  return T2W_OK;
}

size_t t2w_enc_workspace_bytes(const t2w_encoder* e, const t2w_enc_batch* b) {
  if (!e || !b) return 0;
  t2w_encoder* m = const_cast<t2w_encoder*>(e);
  std::lock_guard<std::mutex> lk(m->mu);
  EncPlan pl;
  if (plan_call(m, *b, false, pl)) return 0;
  return layout_of(e->cfg, pl).total;
}

int t2w_encode(t2w_encoder* e, const t2w_enc_batch* b, void* ws, size_t ws_bytes, uint32_t flags, void* stream) {
  if (!e || !b || !ws || !b->mu) return T2W_ERR_INVALID;
  DeviceGuard g(e->device);
  if (!g.ok) return T2W_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lk(e->mu);
  EncPlan pl;
  E_TRY(plan_call(e, *b, true, pl));
  const EncLayout Lo = layout_of(e->cfg, pl);
  // slots taken by the plan, per window in order (returned to the pools if the call fails before it is enqueued)
  std::vector<int32_t> taken1(pl.sc1_slot), taken2(pl.sc2_slot);
  auto give_back = [&]() {
    e->s1.give(taken1.data(), taken1.size());
    e->s2.give(taken2.data(), taken2.size());
  };
  if (ws_bytes < Lo.total || (reinterpret_cast<uintptr_t>(ws) & 255)) {
    give_back();
    return ws_bytes < Lo.total ? T2W_ERR_WORKSPACE : T2W_ERR_INVALID;
  }
  int rc = upload(e, pl, Lo, ws, st);
  if (!rc) {
    const uint64_t key = call_key(pl, ws, b->mu);
    if (e->seen.size() > 4096) e->seen.clear();
    if ((flags & T2W_FLAG_GRAPH) && (e->graphs.count(key) || ++e->seen[key] >= 2)) {
      rc = replay(e, key, st, [&](cudaStream_t cs) { return run_call(e, pl, Lo, ws, b->mu, cs); });
    } else {
      rc = run_call(e, pl, Lo, ws, b->mu, st);
      if (!rc) ++e->n_eager;
    }
  }
  if (rc) {
    // launches may already be enqueued: the new slots stay unused but are given back only once they are idle
    cudaStreamSynchronize(st);
    give_back();
    return rc;
  }
  size_t f1 = 0, f2 = 0;
  for (int i = 0; i < pl.n; ++i) {
    EncRecord& r = *e->find(b->handle[i]);
    const int T = pl.er[i].T;
    advance(e, r, taken1.data() + f1, T);
    advance2(e, r, taken2.data() + f2, 2 * T);
    f1 += T;
    f2 += 2 * T;
  }
  return T2W_OK;
}

int t2w_enc_counts(const t2w_encoder* e, int64_t* replays, int64_t* captures, int64_t* eager) {
  if (!e) return T2W_ERR_INVALID;
  if (replays) *replays = e->n_replays;
  if (captures) *captures = e->n_captures;
  if (eager) *eager = e->n_eager;
  return T2W_OK;
}

int t2w_enc_check(t2w_encoder* e) {
  if (!e) return T2W_ERR_INVALID;
  DeviceGuard g(e->device);
  int v = 0;
  E_CUDA(cudaMemcpy(&v, e->err, 4, cudaMemcpyDeviceToHost));
  if (v) {
    const int z = 0;
    E_CUDA(cudaMemcpy(e->err, &z, 4, cudaMemcpyHostToDevice));
  }
  return v;
}

int t2w_enc_relattn(const void* qkv4, int32_t rows, int32_t heads, const void* pool, int32_t pool_rows, const void* pos,
                    int32_t max_frames, int32_t n_seq, const int32_t* q_row, const int32_t* T, const int32_t* K,
                    const int32_t* kv_off, const int32_t* kv_idx, int32_t n_idx, void* out, void* stream) {
  if (!qkv4 || !pool || !pos || !out || heads <= 0 || rows <= 0 || pool_rows <= 0 || max_frames <= 0 || n_seq < 0 ||
      (n_seq && (!q_row || !T || !K || !kv_off || !kv_idx)) || n_idx < 0)
    return T2W_ERR_INVALID;
  std::vector<RelWork> work;
  for (int s = 0; s < n_seq; ++s) {
    if (T[s] <= 0 || K[s] < T[s] || K[s] > max_frames || T[s] > max_frames || q_row[s] < 0 ||
        (int64_t)q_row[s] + T[s] > rows || kv_off[s] < 0 || (int64_t)kv_off[s] + K[s] > n_idx)
      return T2W_ERR_INVALID;
    for (int j = 0; j < K[s]; ++j)
      if (kv_idx[kv_off[s] + j] < 0 || kv_idx[kv_off[s] + j] >= pool_rows) return T2W_ERR_INVALID;
    for (int q = 0; q < T[s]; q += 128) work.push_back(RelWork{q_row[s] + q, q, T[s], K[s], kv_off[s]});
  }
  if (work.empty()) return T2W_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  E_CUDA(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;
  const int H = heads * 64;
  CUtensorMap tq, tp;
  if (!make_relattn_tmaps(&tq, &tp, qkv4, rows, H, pos, max_frames)) return T2W_ERR_INVALID;
  RelWork* dw = nullptr;
  int* di = nullptr;
  E_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&dw), work.size() * sizeof(RelWork), st));
  E_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&di), (size_t)std::max(n_idx, 1) * 4, st));
  E_CUDA(cudaMemcpyAsync(dw, work.data(), work.size() * sizeof(RelWork), cudaMemcpyHostToDevice, st));
  if (n_idx) E_CUDA(cudaMemcpyAsync(di, kv_idx, (size_t)n_idx * 4, cudaMemcpyHostToDevice, st));
  RelArgs a;
  a.work = dw;
  a.n_work = (int)work.size();
  a.heads = heads;
  a.pool = static_cast<const __nv_bfloat16*>(pool);
  a.pool_ld = 2 * H;
  a.kv_idx = di;
  a.r0 = max_frames - 1;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = H;
  a.scale_log2 = (float)(1.4426950408889634 / 8.0);
  const int rc = launch_relattn(a, tq, tp, st);
  cudaFreeAsync(dw, st);
  cudaFreeAsync(di, st);
  return rc;
}

int t2w_enc_pos_table(const float* w, int32_t H, int32_t max_frames, float max_period, void* pos, void* stream) {
  return launch_pos_table(w, H, max_frames, max_period, static_cast<__nv_bfloat16*>(pos),
                          static_cast<cudaStream_t>(stream));
}

int t2w_enc_ln(const float* x, const float* w, const float* b, float eps, int32_t rows, int32_t C, float* out_f32,
               void* out_bf16, const uint8_t* pad, void* stream) {
  return launch_enc_ln(x, w, b, eps, rows, C, out_f32, static_cast<__nv_bfloat16*>(out_bf16), pad,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"
