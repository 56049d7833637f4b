// The Token2Wav DiT/CFM solver runtime and the C ABI of libt2w_b200.so.
//
// A solver owns its weights (cast to bf16 / re-laid out once at creation, as FastDiT casts them:
// engine/runtime/dit_fast.py:131-145) and every step's adaLN modulation table (computed once on the device by the
// time-embedding kernel, as FastDiT._modulations does on the host: dit_fast.py:157-178).  A solve is planned on the
// host (token rows, pad rows, attention work items), its small index arrays are copied into the caller's workspace,
// and the S-step CFG Euler loop is enqueued on the caller's stream: per step the in_proj GEMM, per block ten kernels
// (LN+mod, QKV GEMM with the q/k norms, attention, proj GEMM + gated residual, LN+mod, conv GEMM, LN+Mish, conv GEMM +
// gated residual, LN+mod, fc1 GEMM + GELU, fc2 GEMM + gated residual; 12 launches), then LN+mod, the final GEMM and the
// fused CFG/Euler kernel.  With T2W_FLAG_GRAPH the whole solve is captured once per (layout, buffers) key into a CUDA
// graph and replayed (the reference replays one graph per solve: dit_fast.py:393-422,470).
//
// Packed row layout (both CFG halves at fixed offsets, as dit_fast.py:19-23 lays its tokens out): the cond half holds
// each stream's segment [2 zero rows | L_i frames]; the uncond half repeats it at row offset half_rows.  The two zero
// rows in front of each segment are the causal convolutions' left padding (the reference's empty conv cache at a
// prompt setup), so a conv tap is a plain row shift and the im2col matrix never exists.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "cache_registry.h"
#include "common.cuh"
#include "kernels.h"

namespace t2w {

static thread_local int g_last_cuda_error = 0;
void set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("T2W_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_tmap_2d_ex(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                     uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || (reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes & 15) || box_rows > 256 ||
      box_cols * (uint32_t)elem_bytes != (uint32_t)swizzle_bytes)
    return false;
  const CUtensorMapDataType dt = elem_bytes == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (sw == CU_TENSOR_MAP_SWIZZLE_NONE) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                  uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols) {
  return make_tmap_2d_ex(map, base, elem_bytes, rows, cols, pitch_bytes, box_rows, box_cols, 128);
}

}  // namespace t2w

using namespace t2w;

namespace {

#define T2W_CUDA(call)                   \
  do {                                   \
    cudaError_t e_ = (call);             \
    if (e_ != cudaSuccess) {             \
      set_cuda_error(e_);                \
      return T2W_ERR_CUDA;               \
    }                                    \
  } while (0)
#define T2W_TRY(call)       \
  do {                      \
    int rc_ = (call);       \
    if (rc_) return rc_;    \
  } while (0)

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct BlockW {
  // bf16 path
  __nv_bfloat16 *qkv = nullptr, *proj = nullptr, *c1 = nullptr, *c2 = nullptr, *fc1 = nullptr, *fc2 = nullptr;
  float *b_qkv, *qn_w, *qn_b, *kn_w, *kn_b, *b_proj, *b_c1, *cln_w, *cln_b, *b_c2, *b_fc1, *b_fc2;
  WeightMaps tm_qkv, tm_proj, tm_c1, tm_c2, tm_fc1, tm_fc2;
  // FP8 path: e4m3 matrices (same [N, Kt] layouts) with their per-1x128-block scale atoms, and 256-row TMA maps
  uint8_t* w8[6] = {};
  uint8_t* sf8[6] = {};
  CUtensorMap t8[6];
};
enum { W8_QKV, W8_PROJ, W8_C1, W8_C2, W8_FC1, W8_FC2 };

struct Plan {
  int n_streams = 0, n_tok = 0, half_rows = 0, rows = 0, n_work = 0;
  std::vector<int> tok_row, tok_stream;
  std::vector<uint8_t> pad;
  std::vector<AttnWork> work;
  uint64_t key = 0;
  // slot-pool (steady-state) solves only: gathered attention key lists, conv rows, and the new keys' (row, slot)
  bool slots = false;
  bool pair_attn = false;  // every window within 64 frames: attention in its paired form
  std::vector<int> kv_idx, tok_qrow, tok_slot;
  std::vector<ConvRow> conv_rows;
  // solves over library-kept caches: x0 gathered on the device from the flow's noise at column tok_col[token]
  bool gather = false;
  std::vector<int> tok_col;
};

// The flow's fixed noise a gathered x0 is read from ([mel, frames] fp32) and its temperature.
struct NoiseSrc {
  const float* noise = nullptr;
  int frames = 0;
  float temperature = 1.f;
};

struct WsLayout {
  size_t hx, h, a, qkv, o, y, c1, f, dphi, x, pad, tok_row, tok_stream, work;
  // FP8 path: e4m3 activations and their scale atoms (sf_h: bytes of one layout for a [rows + 128, hidden] matrix)
  size_t a8, sfa, o8, sfo, c18, sfc1, f8, sff, sf_h, sf_f;
  // slot-pool solves: device copies of the plan's key lists, conv rows and new-key scatter lists
  size_t kv_idx, conv_rows, tok_qrow, tok_slot;
  // solves over library-kept caches: the gathered x0 [n_tok, mel] and each token's noise column
  size_t x0g, tok_col;
  // the block of index arrays uploaded per plan (pad .. tok_col)
  size_t meta, meta_bytes;
  // completion counters of the GEMMs whose following row kernel starts early: [step][block][4][rows / 128]
  size_t done;
  size_t total;
};

uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h * 0xff51afd7ed558ccdull;
}

}  // namespace

struct t2w_solver {
  t2w_config cfg{};
  int precision = T2W_PREC_BF16;
  int device = 0;
  void* arena = nullptr;
  __nv_bfloat16 *w_in = nullptr, *w_fin = nullptr;
  float *b_in = nullptr, *b_fin = nullptr;
  float *mods = nullptr, *final_mods = nullptr, *dts_dev = nullptr;
  std::vector<float> dts;
  std::vector<BlockW> blk;
  WeightMaps tm_in{}, tm_fin{};
  int* err = nullptr;
  cudaStream_t cap_stream = nullptr;
  // cached solve graphs: the executable and an event recorded after its latest launch (an evicted graph may still be
  // running on another caller stream; its event is waited on before the executable is destroyed)
  struct CachedGraph {
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t done = nullptr;
  };
  std::unordered_map<uint64_t, CachedGraph> graphs;
  std::unordered_map<uint64_t, int> slot_seen;  // slot-solve graph keys seen so far (captured on the second call)
  std::unordered_map<uintptr_t, uint64_t> ws_meta;  // workspace -> plan key of the index arrays it holds
  std::vector<cudaEvent_t> prof_events;
  int64_t n_replays = 0, n_captures = 0, n_eager = 0;
  // pinned host images of the plans' index arrays, rotated between uploads
  static constexpr int kStaging = 4;
  struct Staging {
    void* host = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;
    bool used = false;
  };
  Staging staging[kStaging];
  int staging_next = 0;
};

// Device pools of the steady-state solve (one per solver and device): K/V slots per (step, block) and conv-cache row
// slots per (step, block).
struct t2w_slots {
  int device = 0, n_slots = 0, n_rowslots = 0, n_sb = 0, H = 0;
  // the caches kept by the library (handles, key orders, slot allocation) and the lock its entry points take
  t2w::CacheRegistry reg;
  std::mutex mu;
  __nv_bfloat16* kv = nullptr;   // [n_sb][n_slots][2 H]
  __nv_bfloat16* cnn = nullptr;  // [n_sb][n_rowslots][2 convs][2 frames][H]
  long long kv_sb() const { return (long long)n_slots * 2 * H; }
  long long cnn_slot() const { return 4ll * H; }
  long long cnn_sb() const { return (long long)n_rowslots * 4 * H; }
};

namespace {

bool valid_cfg(const t2w_config& c) {
  return c.mel > 0 && c.mel % 16 == 0 && c.mel <= 128 && c.head_dim == 64 && c.heads > 0 &&
         c.hidden == c.heads * c.head_dim && c.hidden % 128 == 0 && c.hidden <= 1024 && c.ffn % 128 == 0 &&
         c.depth > 0 && c.steps > 0 && c.steps <= 16 && c.freq_dim > 0 && c.freq_dim % 2 == 0 &&
         gemm_n_supported(3 * c.hidden) && gemm_n_supported(c.ffn) && gemm_n_supported(c.hidden) &&
         (4 * c.mel) % 64 == 0 && (c.mel == 80 || gemm_n_supported(c.mel));
}

bool make_plan(const t2w_config& c, int n, const int* P, const int* T, Plan& pl) {
  if (n <= 0 || !P || !T) return false;
  pl = Plan();
  pl.n_streams = n;
  uint64_t key = mix(0, (uint64_t)n);
  long long half = 0;
  for (int i = 0; i < n; ++i) {
    if (P[i] < 0 || T[i] < 0 || P[i] + T[i] <= 0) return false;
    half += 2 + P[i] + T[i];
    pl.n_tok += P[i] + T[i];
    key = mix(mix(key, (uint64_t)P[i]), (uint64_t)T[i]);
  }
  half = (half + 7) / 8 * 8;
  if (2 * half + 128 > (1ll << 30)) return false;
  pl.half_rows = (int)half;
  pl.rows = (int)((2 * half + 127) / 128 * 128);
  pl.pad.assign(pl.rows, 1);
  pl.tok_row.resize(pl.n_tok);
  pl.tok_stream.resize(pl.n_tok);
  int tok = 0, row = 0;
  for (int i = 0; i < n; ++i) {
    const int L = P[i] + T[i];
    row += 2;
    for (int t = 0; t < L; ++t) {
      pl.tok_row[tok] = row + t;
      pl.tok_stream[tok] = i;
      pl.pad[row + t] = 0;
      pl.pad[row + t + half] = 0;
      ++tok;
    }
    for (int hh = 0; hh < 2; ++hh)
      for (int q = 0; q < L; q += 128) pl.work.push_back(AttnWork{row + hh * (int)half + q, row + hh * (int)half, q, P[i], L});
    row += L;
  }
  pl.n_work = (int)pl.work.size();
  pl.key = mix(key, (uint64_t)c.hidden);
  return true;
}

// Steady-state plan: one window of T[i] frames per request against its cached keys.  Rows as the packed plan with no
// prompt part: per CFG half, per request [2 conv-cache rows | T[i] window rows].  CFG row r (cond rows 0..n-1, then
// uncond rows) attends the kv_len[r] pool slots of its list (its cached keys, then its T[i] new slots, which the QKV
// output is scattered into) and reads / writes conv-cache row slots rd[r] / wr[r].
bool make_plan_slots(const t2w_config& c, int n, const int* T, const int* kv_len, const int* kv_idx, const int* rd,
                     const int* wr, int n_slots, int n_rowslots, Plan& pl) {
  if (n <= 0 || !T || !kv_len || !kv_idx || !rd || !wr) return false;
  std::vector<int> P0(n, 0);
  for (int i = 0; i < n; ++i)
    if (T[i] <= 0) return false;
  if (!make_plan(c, n, P0.data(), T, pl)) return false;
  pl.slots = true;
  pl.work.clear();
  long long off = 0;
  std::vector<long long> kv_off(2 * n);
  for (int r = 0; r < 2 * n; ++r) {
    const int i = r % n;
    if (kv_len[r] < T[i] || rd[r] < 0 || rd[r] >= n_rowslots || wr[r] < 0 || wr[r] >= n_rowslots) return false;
    kv_off[r] = off;
    off += kv_len[r];
  }
  if (off > (1ll << 30)) return false;
  pl.kv_idx.assign(kv_idx, kv_idx + off);
  for (long long j = 0; j < off; ++j)
    if (pl.kv_idx[j] < 0 || pl.kv_idx[j] >= n_slots) return false;
  int row = 0;
  for (int i = 0; i < n; ++i) {
    row += 2;
    for (int hh = 0; hh < 2; ++hh) {
      const int r = hh * n + i, seg = row + hh * pl.half_rows;
      for (int q = 0; q < T[i]; q += 128) pl.work.push_back(AttnWork{seg + q, (int)kv_off[r], q, T[i], kv_len[r]});
      pl.conv_rows.push_back(ConvRow{seg, T[i], rd[r], wr[r]});
      for (int t = 0; t < T[i]; ++t) {
        pl.tok_qrow.push_back(seg + t);
        pl.tok_slot.push_back(pl.kv_idx[kv_off[r] + kv_len[r] - T[i] + t]);
      }
    }
    row += T[i];
  }
  pl.n_work = (int)pl.work.size();
  // Windows of up to 64 frames: two (window, head) items share each 128-row attention tile (measured on steady calls
  // of 32 and 64 windows of 50 frames; T2W_ATTN_PAIR=0 keeps one item per tile).
  static const bool pair_ok = [] {
    const char* e = getenv("T2W_ATTN_PAIR");
    return !(e && e[0] == '0');
  }();
  pl.pair_attn = pair_ok;
  for (const AttnWork& w : pl.work)
    if (w.P - w.q_pos > 64) pl.pair_attn = false;
  return true;
}

WsLayout layout(const t2w_config& c, const Plan& pl, bool fp8) {
  WsLayout w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t R = (size_t)pl.rows, H = (size_t)c.hidden;
  w.hx = take(R * 4 * c.mel * 2);
  w.h = take(R * H * 4);
  w.a = take(R * H * 2);
  w.qkv = take(R * 3 * H * 2);
  w.o = take(R * H * 2);
  w.y = take(R * H * 2);
  w.c1 = take(R * H * 2);
  w.f = take(R * (size_t)c.ffn * 2);
  w.dphi = take(R * (size_t)c.mel * 4);
  w.x = take((size_t)pl.n_tok * c.mel * 4);
  w.done = take((size_t)c.steps * c.depth * 4 * (pl.rows / 128) * sizeof(int));
  if (pl.gather) w.x0g = take((size_t)pl.n_tok * c.mel * 4);
  // the plan's index arrays, packed in one block (16-byte aligned entries) that one host-to-device copy fills
  w.meta = off;
  auto put = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 15) & ~size_t(15);
    return o;
  };
  w.pad = put(R);
  w.tok_row = put((size_t)pl.n_tok * 4);
  w.tok_stream = put((size_t)pl.n_tok * 4);
  w.work = put((size_t)pl.n_work * sizeof(AttnWork));
  if (pl.slots) {
    w.kv_idx = put(pl.kv_idx.size() * 4);
    w.conv_rows = put(pl.conv_rows.size() * sizeof(ConvRow));
    w.tok_qrow = put(pl.tok_qrow.size() * 4);
    w.tok_slot = put(pl.tok_slot.size() * 4);
  }
  if (pl.gather) w.tok_col = put(pl.tok_col.size() * 4);
  w.meta_bytes = off - w.meta;
  off = align256(off);
  if (fp8) {
    // the row-shifted scale layouts hold rows up to rows + 1: one spare row tile
    w.sf_h = align256(gemm8_sf_bytes(pl.rows + 128, c.hidden));
    w.sf_f = align256(gemm8_sf_bytes(pl.rows + 128, c.ffn));
    w.a8 = take(R * H);
    w.sfa = take(3 * w.sf_h);
    w.o8 = take(R * H);
    w.sfo = take(w.sf_h);
    w.c18 = take(R * H);
    w.sfc1 = take(3 * w.sf_h);
    w.f8 = take(R * (size_t)c.ffn);
    w.sff = take(w.sf_f);
  }
  w.total = off;
  return w;
}

template <class T>
T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

bool weight_map(WeightMaps* m, const void* w, int N, int Ktot) { return make_weight_maps(m, w, N, Ktot); }

// Optional per-launch timing: an event before every launch (and one after the last) on the solve's stream.
struct Prof {
  std::vector<cudaEvent_t>* events = nullptr;
  std::vector<int> cls;
  int tick(int c, cudaStream_t st) {
    if (!events) return T2W_OK;
    if (events->size() <= cls.size()) {
      cudaEvent_t e;
      T2W_CUDA(cudaEventCreate(&e));
      events->push_back(e);
    }
    T2W_CUDA(cudaEventRecord((*events)[cls.size()], st));
    cls.push_back(c);
    return T2W_OK;
  }
};

// Enqueue one whole solve (no host synchronisation, graph-capturable).
int enqueue_solve(t2w_solver* s, const Plan& pl, const t2w_batch& b, void* ws, cudaStream_t st, Prof* prof = nullptr,
                  const t2w_slots* sp = nullptr, const NoiseSrc* nsrc = nullptr) {
  Prof none;
  Prof& P = prof ? *prof : none;
  const t2w_config& c = s->cfg;
  const WsLayout L = layout(c, pl, s->precision == T2W_PREC_FP8);
  const int H = c.hidden, R = pl.rows, mel = c.mel, F = c.ffn;
  __nv_bfloat16* hx = at<__nv_bfloat16>(ws, L.hx);
  float* h = at<float>(ws, L.h);
  __nv_bfloat16* a = at<__nv_bfloat16>(ws, L.a);
  __nv_bfloat16* qkv = at<__nv_bfloat16>(ws, L.qkv);
  __nv_bfloat16* o = at<__nv_bfloat16>(ws, L.o);  // attention output, then the first conv's pre-norm output
  __nv_bfloat16* y = at<__nv_bfloat16>(ws, L.y);  // proj / conv2 / fc2 output, added into h by the next norm
  __nv_bfloat16* c1 = at<__nv_bfloat16>(ws, L.c1);
  __nv_bfloat16* f = at<__nv_bfloat16>(ws, L.f);
  float* dphi = at<float>(ws, L.dphi);
  float* x = at<float>(ws, L.x);
  const uint8_t* pad = at<uint8_t>(ws, L.pad);
  const int* tok_row = at<int>(ws, L.tok_row);
  const int* tok_stream = at<int>(ws, L.tok_stream);
  const AttnWork* work = at<AttnWork>(ws, L.work);

  // Operand maps (128-row boxes of 64 bf16 columns) and output maps of the GEMM epilogues (32-row boxes, one epilogue
  // warp's rows: 64 bf16 or 32 fp32 columns).
  CUtensorMap tm_hx, tm_a, tm_o, tm_c1, tm_f;
  CUtensorMap st_o, st_y, st_c1, st_f, st_qkv, st_h;
  if (!make_tmap_2d(&tm_hx, hx, 2, R, 4 * mel, 4 * mel * 2, 128, 64) || !make_tmap_2d(&tm_a, a, 2, R, H, H * 2, 128, 64) ||
      !make_tmap_2d(&tm_o, o, 2, R, H, H * 2, 128, 64) || !make_tmap_2d(&tm_c1, c1, 2, R, H, H * 2, 128, 64) ||
      !make_tmap_2d(&tm_f, f, 2, R, F, F * 2, 128, 64) || !make_tmap_2d(&st_o, o, 2, R, H, H * 2, 32, 64) ||
      !make_tmap_2d(&st_y, y, 2, R, H, H * 2, 32, 64) || !make_tmap_2d(&st_c1, c1, 2, R, H, H * 2, 32, 64) ||
      !make_tmap_2d(&st_f, f, 2, R, F, F * 2, 32, 64) || !make_tmap_2d(&st_qkv, qkv, 2, R, 3 * H, 3 * H * 2, 32, 64) ||
      !make_tmap_2d(&st_h, h, 4, R, H, H * 4, 32, 32))
    return T2W_ERR_INVALID;
  CUtensorMap tm_att_q, tm_att_kv, tm_att_pair;
  if (!make_attn_tmaps(&tm_att_q, &tm_att_kv, qkv, R, c.heads)) return T2W_ERR_INVALID;
  if (pl.pair_attn && !make_attn_pair_tmap(&tm_att_pair, qkv, R, c.heads)) return T2W_ERR_INVALID;
  const bool fp8 = s->precision == T2W_PREC_FP8;
  if (pl.slots && (!sp || fp8)) return T2W_ERR_UNSUPPORTED;  // the slot-pool solve runs the bf16 path
  const int* kv_idx_d = pl.slots ? at<int>(ws, L.kv_idx) : nullptr;
  const ConvRow* conv_rows_d = pl.slots ? at<ConvRow>(ws, L.conv_rows) : nullptr;
  const int* tok_qrow_d = pl.slots ? at<int>(ws, L.tok_qrow) : nullptr;
  const int* tok_slot_d = pl.slots ? at<int>(ws, L.tok_slot) : nullptr;
  const int n_conv_rows = (int)pl.conv_rows.size(), n_new = (int)pl.tok_slot.size();
  uint8_t *a8 = nullptr, *sfa = nullptr, *o8 = nullptr, *sfo = nullptr, *c18 = nullptr, *sfc1 = nullptr, *f8 = nullptr,
          *sff = nullptr;
  CUtensorMap t8_a, t8_o, t8_c1, t8_f, st8_f;
  if (fp8) {
    a8 = at<uint8_t>(ws, L.a8);
    sfa = at<uint8_t>(ws, L.sfa);
    o8 = at<uint8_t>(ws, L.o8);
    sfo = at<uint8_t>(ws, L.sfo);
    c18 = at<uint8_t>(ws, L.c18);
    sfc1 = at<uint8_t>(ws, L.sfc1);
    f8 = at<uint8_t>(ws, L.f8);
    sff = at<uint8_t>(ws, L.sff);
    if (!make_tmap_2d(&t8_a, a8, 1, R, H, H, 128, 128) || !make_tmap_2d(&t8_o, o8, 1, R, H, H, 128, 128) ||
        !make_tmap_2d(&t8_c1, c18, 1, R, H, H, 128, 128) || !make_tmap_2d(&t8_f, f8, 1, R, F, F, 128, 128) ||
        !make_tmap_2d_ex(&st8_f, f8, 1, R, F, F, 32, 64, 64))
      return T2W_ERR_INVALID;
    // scale bytes 127 (= 1) wherever no kernel writes (rows before 0 of the shifted layouts, pad rows of o8)
    T2W_CUDA(cudaMemsetAsync(sfa, 127, 3 * L.sf_h, st));
    T2W_CUDA(cudaMemsetAsync(sfc1, 127, 3 * L.sf_h, st));
    T2W_CUDA(cudaMemsetAsync(sfo, 127, L.sf_h, st));
    T2W_CUDA(cudaMemsetAsync(o8, 0, (size_t)R * H, st));
  }
  RowOut out_a = row_out_bf16(a), out_c1 = row_out_bf16(c1);
  if (fp8) {
    out_a.out = a8;
    out_a.sf = sfa;
    out_a.n_layouts = 3;
    out_a.layout_bytes = (long long)L.sf_h;
    out_c1.out = c18;
    out_c1.sf = sfc1;
    out_c1.n_layouts = 3;
    out_c1.layout_bytes = (long long)L.sf_h;
  }
  // an FP8 GEMM of the block: A8 with its atoms, W8 of block weight `wi`
  auto g8 = [&](const BlockW& w, int wi, const uint8_t* A8, const uint8_t* sf, int layouts, int N, int K, int taps,
                int epi, void* out, int ldo, const float* bias) {
    Gemm8Args a;
    a.A8 = A8;
    a.lda = K;
    a.rows_a = R;
    a.sfa = sf;
    a.sfa_layout = (long long)L.sf_h;
    a.sfa_layouts = layouts;
    a.W8 = w.w8[wi];
    a.sfw = w.sf8[wi];
    a.bias = bias;
    a.M = R;
    a.N = N;
    a.K = K;
    a.taps = taps;
    a.tap_row0 = taps == 3 ? -2 : 0;
    a.epi = epi;
    a.out = out;
    a.ldo = ldo;
    a.err = s->err;
    return a;
  };

  T2W_CUDA(cudaMemsetAsync(hx, 0, (size_t)R * 4 * mel * 2, st));
  // Attention writes only sequence rows; the pad rows of its output buffer must hold finite values (zero here, later
  // finite conv outputs), or the proj GEMM carries workspace garbage into pad rows of h, and a NaN there reaches the
  // masked keys of the next attention, where 0 * NaN poisons the P V product.
  T2W_CUDA(cudaMemsetAsync(o, 0, (size_t)R * H * 2, st));
  int* done_all = at<int>(ws, L.done);
  const int mblocks = R / 128;
  T2W_CUDA(cudaMemsetAsync(done_all, 0, (size_t)c.steps * c.depth * 4 * mblocks * sizeof(int), st));
  // the N = H GEMMs (proj, conv1, conv2, fc2) publish per-block completion; the row kernel after each waits per block
  const int done_target = 8 * (H / gemm_block_n_for(H, R, T2W_EPI_BF16));
  T2W_TRY(P.tick(T2W_KC_PACK, st));
  if (pl.gather) {  // x0 from the flow's noise at each request's cache length, into the workspace (b.x0 points there)
    if (!nsrc || b.x0 != at<float>(ws, L.x0g)) return T2W_ERR_INVALID;
    T2W_TRY(launch_noise_x0(nsrc->noise, nsrc->frames, mel, at<int>(ws, L.tok_col), pl.n_tok, nsrc->temperature,
                            at<float>(ws, L.x0g), st));
  }
  T2W_TRY(launch_pack(b.x0, b.mu, b.cond, b.spk, tok_row, tok_stream, pl.n_tok, mel, pl.half_rows, hx, 4 * mel, x, st));

  GemmArgs g;
  g.rows_a = R;
  g.M = R;
  g.err = s->err;
  AttnArgs at_args;
  at_args.qkv = qkv;
  at_args.rows = R;
  at_args.heads = c.heads;
  at_args.work = work;
  at_args.n_work = pl.n_work;
  at_args.out = o;
  at_args.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)c.head_dim));
  at_args.err = s->err;

  for (int step = 0; step < c.steps; ++step) {
    g = GemmArgs();
    g.rows_a = R;
    g.M = R;
    g.err = s->err;
    g.A = hx; g.lda = 4 * mel; g.W = s->w_in; g.bias = s->b_in; g.N = H; g.K = 4 * mel; g.epi = T2W_EPI_F32;
    g.out = h; g.ldo = H;
    T2W_TRY(P.tick(T2W_KC_GEMM_IN, st));
    T2W_TRY(launch_gemm(g, st, &tm_hx, &s->tm_in, &st_h));
    // The gated residual of each branch (h += g * y) is applied by the norm that follows it (add_ln_mod), as the
    // reference's fused_residual path does (dit_fast.py:306-344); the MLP's pending (g, y) is added by the next block's
    // first norm or by the final layer's norm.  bf16 path, attention branch: the proj GEMM's epilogue adds
    // g * (acc + bias) to h itself (T2W_EPI_RESID, a TMA reduce-add in L2) and the norm after it reads h alone.  proj
    // has K = 512, so its second round of tiles is short and that norm sat on the critical path (measured at config 2:
    // norm 1.32 -> 0.48 ms, proj 2.14 -> 2.82 ms per solve).  After conv2 and fc2 (K = 1536 / 2048) the norm of the
    // early row blocks hides under the GEMM's last round, while the fp32 reduce lengthens the last tile's epilogue:
    // there the same change cost 0.2 ms each, so they keep the bf16 output.
    const float* pend_g = nullptr;
    const __nv_bfloat16* pend_y = nullptr;
    int* pend_done = nullptr;
    for (int bi = 0; bi < c.depth; ++bi) {
      const BlockW& w = s->blk[bi];
      const float* M = s->mods + ((size_t)step * c.depth + bi) * 9 * H;
      const float *sh_a = M, *sc_a = M + H, *g_a = M + 2 * H, *sh_m = M + 3 * H, *sc_m = M + 4 * H, *g_m = M + 5 * H;
      const float *sh_c = M + 6 * H, *sc_c = M + 7 * H, *g_c = M + 8 * H;
      int* dn = done_all + ((size_t)step * c.depth + bi) * 4 * mblocks;  // proj, conv1, conv2, fc2
      // each norm kernel prefetches the weights of the GEMM after it into L2 (HBM-resident: all blocks' weights exceed
      // L2); attention prefetches proj's, and fc1 fc2's as its CTAs start their last tile
      auto waits = [&](int* f, const void* pf = nullptr, size_t pf_bytes = 0, const void* pf2 = nullptr,
                       size_t pf2_bytes = 0) {
        RowWait r;
        r.flags = f;
        r.target = done_target;
        r.err = s->err;
        r.pf = pf;
        r.pf_bytes = (unsigned)pf_bytes;
        r.pf2 = pf2;
        r.pf2_bytes = (unsigned)pf2_bytes;
        return r;
      };
      const size_t wb_hh = (size_t)H * H * 2, wb_conv = 3 * wb_hh, wb_qkv = 3 * wb_hh, wb_mlp = (size_t)F * H * 2;
      if (fp8) {
        // attention branch
        T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
        T2W_TRY(launch_add_ln_mod(h, pend_y, pend_g, sh_a, sc_a, c.eps_block, R, H, out_a, nullptr, st,
                                  waits(nullptr, w.w8[W8_QKV], (size_t)3 * H * H)));
        Gemm8Args q = g8(w, W8_QKV, a8, sfa, 3, 3 * H, H, 1, T2W_EPI_QKV, qkv, 3 * H, w.b_qkv);
        q.qn_w = w.qn_w; q.qn_b = w.qn_b; q.kn_w = w.kn_w; q.kn_b = w.kn_b; q.qk_eps = c.eps_qk;
        T2W_TRY(P.tick(T2W_KC_GEMM_QKV, st));
        T2W_TRY(launch_gemm8(q, st, &t8_a, &w.t8[W8_QKV], &st_qkv));
        AttnArgs at8 = at_args;
        at8.pf = w.w8[W8_PROJ];
        at8.pf_bytes = (unsigned)((size_t)H * H);
        at8.out = o8;
        at8.out_sf = sfo;
        T2W_TRY(P.tick(T2W_KC_ATTN, st));
        T2W_TRY(launch_attn(at8, st, &tm_att_q, &tm_att_kv));
        T2W_TRY(P.tick(T2W_KC_GEMM_PROJ, st));
        T2W_TRY(launch_gemm8(g8(w, W8_PROJ, o8, sfo, 1, H, H, 1, T2W_EPI_BF16, y, H, w.b_proj), st, &t8_o,
                             &w.t8[W8_PROJ], &st_y));
        // causal conv branch
        T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
        T2W_TRY(launch_add_ln_mod(h, y, g_a, sh_c, sc_c, c.eps_block, R, H, out_a, pad, st,
                                  waits(nullptr, w.w8[W8_C1], (size_t)3 * H * H)));
        T2W_TRY(P.tick(T2W_KC_GEMM_CONV1, st));
        T2W_TRY(launch_gemm8(g8(w, W8_C1, a8, sfa, 3, H, H, 3, T2W_EPI_BF16, o, H, w.b_c1), st, &t8_a, &w.t8[W8_C1],
                             &st_o));
        T2W_TRY(P.tick(T2W_KC_LN_MISH, st));
        T2W_TRY(launch_ln_mish(o, w.cln_w, w.cln_b, c.eps_conv, R, H, out_c1, pad, st,
                               waits(nullptr, w.w8[W8_C2], (size_t)3 * H * H)));
        T2W_TRY(P.tick(T2W_KC_GEMM_CONV2, st));
        T2W_TRY(launch_gemm8(g8(w, W8_C2, c18, sfc1, 3, H, H, 3, T2W_EPI_BF16, y, H, w.b_c2), st, &t8_c1,
                             &w.t8[W8_C2], &st_y));
        // MLP branch: fc1's epilogue quantises GELU's output for fc2
        T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
        T2W_TRY(launch_add_ln_mod(h, y, g_c, sh_m, sc_m, c.eps_block, R, H, out_a, nullptr, st,
                                  waits(nullptr, w.w8[W8_FC1], (size_t)F * H)));
        Gemm8Args f1 = g8(w, W8_FC1, a8, sfa, 3, F, H, 1, T2W_EPI_GELU_FP8, f8, F, w.b_fc1);
        f1.out_sf = sff;
        f1.pf = w.w8[W8_FC2];  // fc2's e4m3 weights, as fc1's CTAs start their last tile
        f1.pf_bytes = (unsigned)((size_t)F * H);
        T2W_TRY(P.tick(T2W_KC_GEMM_FC1, st));
        T2W_TRY(launch_gemm8(f1, st, &t8_a, &w.t8[W8_FC1], &st8_f));
        Gemm8Args f2 = g8(w, W8_FC2, f8, sff, 1, H, F, 1, T2W_EPI_BF16, y, H, w.b_fc2);
        f2.sfa_layout = (long long)L.sf_f;
        T2W_TRY(P.tick(T2W_KC_GEMM_FC2, st));
        T2W_TRY(launch_gemm8(f2, st, &t8_f, &w.t8[W8_FC2], &st_y));
        pend_g = g_m;
        pend_y = y;
        pend_done = nullptr;
        continue;
      }
      // attention branch
      T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
      T2W_TRY(launch_add_ln_mod(h, pend_y, pend_g, sh_a, sc_a, c.eps_block, R, H, row_out_bf16(a), nullptr, st,
                                waits(pend_done, w.qkv, wb_qkv)));
      GemmArgs q = GemmArgs();
      q.rows_a = R; q.M = R; q.err = s->err;
      q.A = a; q.lda = H; q.W = w.qkv; q.bias = w.b_qkv; q.N = 3 * H; q.K = H; q.epi = T2W_EPI_QKV; q.out = qkv; q.ldo = 3 * H;
      q.qn_w = w.qn_w; q.qn_b = w.qn_b; q.kn_w = w.kn_w; q.kn_b = w.kn_b; q.qk_eps = c.eps_qk;
      T2W_TRY(P.tick(T2W_KC_GEMM_QKV, st));
      T2W_TRY(launch_gemm(q, st, &tm_a, &w.tm_qkv, &st_qkv));
      const int sb = step * c.depth + bi;
      AttnArgs at_use = at_args;
      at_use.pf = w.proj;
      at_use.pf_bytes = (unsigned)wb_hh;
      if (pl.slots) {  // the window's new keys into their slots; attention gathers every row's key list
        __nv_bfloat16* kvp = sp->kv + sb * sp->kv_sb();
        T2W_TRY(launch_kv_scatter(qkv, H, tok_qrow_d, tok_slot_d, n_new, kvp, st));
        at_use.pool = kvp;
        at_use.kv_idx = kv_idx_d;
        at_use.pool_ld = 2 * H;
        at_use.pair = pl.pair_attn;
        at_use.tm_q_pair = pl.pair_attn ? &tm_att_pair : nullptr;
      }
      T2W_TRY(P.tick(T2W_KC_ATTN, st));
      T2W_TRY(launch_attn(at_use, st, &tm_att_q, &tm_att_kv));
      GemmArgs pr = GemmArgs();
      pr.rows_a = R; pr.M = R; pr.err = s->err;
      pr.A = o; pr.lda = H; pr.W = w.proj; pr.bias = w.b_proj; pr.N = H; pr.K = H; pr.epi = T2W_EPI_RESID; pr.out = h; pr.ldo = H;
      pr.gate = g_a;
      pr.done_flags = dn;
      T2W_TRY(P.tick(T2W_KC_GEMM_PROJ, st));
      T2W_TRY(launch_gemm(pr, st, &tm_o, &w.tm_proj, &st_h));
      // causal conv branch (norm3 / conv modulations: token2wav_batch.py:107-108); pad rows of its input are zero
      T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
      T2W_TRY(launch_add_ln_mod(h, nullptr, nullptr, sh_c, sc_c, c.eps_block, R, H, row_out_bf16(a), pad, st,
                                waits(dn, w.c1, wb_conv)));
      if (pl.slots)  // cached conv-input frames in front of each window, and the window's last two saved
        T2W_TRY(launch_conv_cache(a, H, conv_rows_d, n_conv_rows, sp->cnn + sb * sp->cnn_sb(), sp->cnn_slot(), st));
      GemmArgs k1 = GemmArgs();
      k1.rows_a = R; k1.M = R; k1.err = s->err;
      k1.A = a; k1.lda = H; k1.W = w.c1; k1.bias = w.b_c1; k1.N = H; k1.K = H; k1.taps = 3; k1.tap_row0 = -2;
      k1.epi = T2W_EPI_BF16; k1.out = o; k1.ldo = H;
      k1.done_flags = dn + mblocks;
      T2W_TRY(P.tick(T2W_KC_GEMM_CONV1, st));
      T2W_TRY(launch_gemm(k1, st, &tm_a, &w.tm_c1, &st_o));
      T2W_TRY(P.tick(T2W_KC_LN_MISH, st));
      T2W_TRY(launch_ln_mish(o, w.cln_w, w.cln_b, c.eps_conv, R, H, row_out_bf16(c1), pad, st,
                             waits(dn + mblocks, w.c2, wb_conv)));
      if (pl.slots)
        T2W_TRY(launch_conv_cache(c1, H, conv_rows_d, n_conv_rows, sp->cnn + sb * sp->cnn_sb() + 2 * H, sp->cnn_slot(), st));
      GemmArgs k2 = GemmArgs();
      k2.rows_a = R; k2.M = R; k2.err = s->err;
      k2.A = c1; k2.lda = H; k2.W = w.c2; k2.bias = w.b_c2; k2.N = H; k2.K = H; k2.taps = 3; k2.tap_row0 = -2;
      k2.epi = T2W_EPI_BF16; k2.out = y; k2.ldo = H;
      k2.done_flags = dn + 2 * mblocks;
      // Large batches: conv2 and fc2 also add their gated residual in the epilogue (TMA reduce-add into h), so the norm
      // after each reads h alone instead of h and y and writing h back: at the target shape (64 x (300 + 50), 704 tiles
      // per N = 512 GEMM) the solve went 109.5 -> 106.4 ms; at config 2 (176 tiles) the longer fp32 epilogue of the
      // last round costs more than the norm saves (29.1 -> 29.5 ms), so below three rounds of tiles they keep bf16 y.
      const bool ra = (long long)mblocks * (H / 256) >= 3ll * num_sms();
      if (ra) {
        k2.epi = T2W_EPI_RESID; k2.out = h; k2.gate = g_c;
      }
      T2W_TRY(P.tick(T2W_KC_GEMM_CONV2, st));
      T2W_TRY(launch_gemm(k2, st, &tm_c1, &w.tm_c2, ra ? &st_h : &st_y));
      // MLP branch
      T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
      T2W_TRY(launch_add_ln_mod(h, ra ? nullptr : y, ra ? nullptr : g_c, sh_m, sc_m, c.eps_block, R, H,
                                row_out_bf16(a), nullptr, st, waits(dn + 2 * mblocks, w.fc1, wb_mlp)));
      GemmArgs f1 = GemmArgs();
      f1.rows_a = R; f1.M = R; f1.err = s->err;
      f1.A = a; f1.lda = H; f1.W = w.fc1; f1.bias = w.b_fc1; f1.N = F; f1.K = H; f1.epi = T2W_EPI_GELU; f1.out = f; f1.ldo = F;
      f1.pf = w.fc2;
      f1.pf_bytes = (unsigned)wb_mlp;
      T2W_TRY(P.tick(T2W_KC_GEMM_FC1, st));
      T2W_TRY(launch_gemm(f1, st, &tm_a, &w.tm_fc1, &st_f));
      GemmArgs f2 = GemmArgs();
      f2.rows_a = R; f2.M = R; f2.err = s->err;
      f2.A = f; f2.lda = F; f2.W = w.fc2; f2.bias = w.b_fc2; f2.N = H; f2.K = F; f2.epi = T2W_EPI_BF16; f2.out = y; f2.ldo = H;
      f2.done_flags = dn + 3 * mblocks;
      if (ra) {
        f2.epi = T2W_EPI_RESID; f2.out = h; f2.gate = g_m;
      }
      T2W_TRY(P.tick(T2W_KC_GEMM_FC2, st));
      T2W_TRY(launch_gemm(f2, st, &tm_f, &w.tm_fc2, ra ? &st_h : &st_y));
      pend_g = ra ? nullptr : g_m;
      pend_y = ra ? nullptr : y;
      pend_done = dn + 3 * mblocks;
    }
    const float* FM = s->final_mods + (size_t)step * 2 * H;
    T2W_TRY(P.tick(T2W_KC_LN_MOD, st));
    RowWait fw;
    fw.flags = pend_done;
    fw.target = done_target;
    fw.err = s->err;
    T2W_TRY(launch_add_ln_mod(h, pend_y, pend_g, FM, FM + H, c.eps_final, R, H, row_out_bf16(a), nullptr, st, fw));
    GemmArgs fin = GemmArgs();
    fin.rows_a = R; fin.M = R; fin.err = s->err;
    fin.A = a; fin.lda = H; fin.W = s->w_fin; fin.bias = s->b_fin; fin.N = mel; fin.K = H; fin.epi = T2W_EPI_F32;
    fin.out = dphi; fin.ldo = mel;
    T2W_TRY(P.tick(T2W_KC_GEMM_FINAL, st));
    T2W_TRY(launch_gemm(fin, st, &tm_a, &s->tm_fin, nullptr));
    const bool last = step == c.steps - 1;
    T2W_TRY(P.tick(T2W_KC_EULER, st));
    T2W_TRY(launch_euler(x, dphi, mel, tok_row, pl.n_tok, mel, pl.half_rows, s->dts[step], c.cfg_rate,
                         last ? nullptr : hx, 4 * mel, last ? b.out : nullptr, st));
  }
  return P.tick(-1, st);  // closing event
}

// Copy the plan's index arrays into the workspace: their image is assembled in a pinned host staging buffer and moved
// by one asynchronous copy (a copy from pageable memory would first synchronise the stream, stalling the host on the
// previous solve).  Staging buffers rotate; one is rewritten only after the copy that last read it has completed.
int upload_meta(t2w_solver* s, const Plan& pl, void* ws, cudaStream_t st) {
  const WsLayout L = layout(s->cfg, pl, s->precision == T2W_PREC_FP8);
  t2w_solver::Staging& sg = s->staging[s->staging_next];
  s->staging_next = (s->staging_next + 1) % t2w_solver::kStaging;
  if (sg.used) T2W_CUDA(cudaEventSynchronize(sg.done));
  if (sg.cap < L.meta_bytes) {
    if (sg.host) cudaFreeHost(sg.host);
    sg.host = nullptr;
    sg.cap = 0;
    const size_t cap = std::max<size_t>(L.meta_bytes + L.meta_bytes / 4, 1 << 16);
    T2W_CUDA(cudaMallocHost(&sg.host, cap));
    sg.cap = cap;
  }
  if (!sg.done) T2W_CUDA(cudaEventCreateWithFlags(&sg.done, cudaEventDisableTiming));
  uint8_t* img = static_cast<uint8_t*>(sg.host);
  auto put = [&](size_t off, const void* src, size_t bytes) {
    if (bytes) std::memcpy(img + (off - L.meta), src, bytes);
  };
  put(L.pad, pl.pad.data(), pl.pad.size());
  put(L.tok_row, pl.tok_row.data(), pl.tok_row.size() * 4);
  put(L.tok_stream, pl.tok_stream.data(), pl.tok_stream.size() * 4);
  put(L.work, pl.work.data(), pl.work.size() * sizeof(AttnWork));
  if (pl.slots) {
    put(L.kv_idx, pl.kv_idx.data(), pl.kv_idx.size() * 4);
    put(L.conv_rows, pl.conv_rows.data(), pl.conv_rows.size() * sizeof(ConvRow));
    put(L.tok_qrow, pl.tok_qrow.data(), pl.tok_qrow.size() * 4);
    put(L.tok_slot, pl.tok_slot.data(), pl.tok_slot.size() * 4);
  }
  if (pl.gather) put(L.tok_col, pl.tok_col.data(), pl.tok_col.size() * 4);
  T2W_CUDA(cudaMemcpyAsync(at<uint8_t>(ws, L.meta), img, L.meta_bytes, cudaMemcpyHostToDevice, st));
  T2W_CUDA(cudaEventRecord(sg.done, st));
  sg.used = true;
  if (pl.slots) {
    s->ws_meta.erase(reinterpret_cast<uintptr_t>(ws));  // slot lists change every call: nothing to reuse
    return T2W_OK;
  }
  s->ws_meta[reinterpret_cast<uintptr_t>(ws)] = pl.key;
  return T2W_OK;
}

// Launch the solve graph cached under `key` on `st`, capturing `enqueue` into it first if there is none.  The capture
// runs on the solver's own stream (the caller's may be the legacy default stream, which cannot be captured); capturing
// executes nothing.  At most kMaxGraphs graphs are kept: past that, one is dropped once its latest launch has finished.
// The solver's (or slot pool's) device is made current for the duration of a call and the caller's restored after it:
// its memory, streams and graphs belong to that device, and a caller that drives several GPUs from one thread may have
// another one current.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) {
      ok = false;
      return;
    }
    if (cur != dev) {
      ok = cudaSetDevice(dev) == cudaSuccess;
      prev = cur;
    }
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
#define T2W_ON_DEVICE(dev)              \
  DeviceGuard t2w_device_guard_(dev);   \
  if (!t2w_device_guard_.ok) return T2W_ERR_CUDA

constexpr size_t kMaxGraphs = 64;
template <class F>
int replay(t2w_solver* s, uint64_t key, cudaStream_t st, F&& enqueue) {
  auto g = s->graphs.find(key);
  if (g == s->graphs.end()) {
    cudaStreamCaptureStatus cs;
    T2W_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;  // the caller is capturing: use flags = 0
    if (s->graphs.size() >= kMaxGraphs) {  // drop one, once its latest launch (on whichever stream) has finished
      auto victim = s->graphs.begin();
      T2W_CUDA(cudaEventSynchronize(victim->second.done));
      cudaGraphExecDestroy(victim->second.exec);
      cudaEventDestroy(victim->second.done);
      s->graphs.erase(victim);
    }
    if (!s->cap_stream) T2W_CUDA(cudaStreamCreateWithFlags(&s->cap_stream, cudaStreamNonBlocking));
    T2W_CUDA(cudaStreamBeginCapture(s->cap_stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue(s->cap_stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(s->cap_stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ec != cudaSuccess) {
      set_cuda_error(ec);
      return T2W_ERR_CUDA;
    }
    t2w_solver::CachedGraph cg;
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
    g = s->graphs.emplace(key, cg).first;
    ++s->n_captures;
  }
  T2W_CUDA(cudaGraphLaunch(g->second.exec, st));
  T2W_CUDA(cudaEventRecord(g->second.done, st));
  ++s->n_replays;
  return T2W_OK;
}

// Varlen attention with a per-call device work list (one entry per 128-query tile of each sequence).
int attn_varlen_alloc(const void* qkv, int rows, int heads, int n_seq, const int32_t* seq_row, const int32_t* seq_len,
                      const int32_t* prompt_len, void* out, uint8_t* out_sf, void* stream) {
  if (!qkv || !out || !seq_row || !seq_len || !prompt_len || n_seq < 0 || heads <= 0) return T2W_ERR_INVALID;
  std::vector<AttnWork> work;
  for (int s = 0; s < n_seq; ++s) {
    if (seq_len[s] <= 0 || prompt_len[s] < 0 || prompt_len[s] > seq_len[s] || seq_row[s] < 0 ||
        (int64_t)seq_row[s] + seq_len[s] > rows)
      return T2W_ERR_INVALID;
    for (int q = 0; q < seq_len[s]; q += 128)
      work.push_back(AttnWork{seq_row[s] + q, seq_row[s], q, prompt_len[s], seq_len[s]});
  }
  if (work.empty()) return T2W_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the work list is copied from a host vector that dies with this call: a capturing stream is refused
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  T2W_CUDA(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;
  AttnWork* d = nullptr;
  T2W_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d), work.size() * sizeof(AttnWork), st));
  T2W_CUDA(cudaMemcpyAsync(d, work.data(), work.size() * sizeof(AttnWork), cudaMemcpyHostToDevice, st));
  AttnArgs a;
  a.qkv = qkv;
  a.rows = rows;
  a.heads = heads;
  a.work = d;
  a.n_work = (int)work.size();
  a.out = out;
  a.out_sf = out_sf;
  a.scale_log2 = (float)(1.4426950408889634 / 8.0);
  const int rc = launch_attn(a, st);
  cudaFreeAsync(d, st);
  return rc;
}

// Enqueue a planned slot-pool solve (eager, or a CUDA graph per launch structure).  The launches depend on the plan's
// sizes and the buffers only: the slot lists, conv rows, work list (and, for gathered x0, the noise columns) are read
// from the workspace, where upload_meta has just put this call's.  A graph per such key, captured the second time the
// key is seen (a key met once, as while caches still grow towards their trimmed length, runs eagerly).
int run_slot_plan(t2w_solver* s, t2w_slots* p, const Plan& pl, const t2w_batch& pb, void* ws, uint32_t flags,
                  cudaStream_t st, const NoiseSrc* nsrc) {
  T2W_TRY(upload_meta(s, pl, ws, st));
  uint64_t key = 0x510750175107ull;
  for (long long v : {(long long)pl.n_streams, (long long)pl.n_tok, (long long)pl.half_rows, (long long)pl.rows,
                      (long long)pl.n_work, (long long)pl.kv_idx.size(), (long long)pl.conv_rows.size(),
                      (long long)pl.tok_slot.size(), (long long)pl.gather, (long long)pl.pair_attn})
    key = mix(key, (uint64_t)v);
  for (const void* q : {(const void*)ws, (const void*)pb.x0, (const void*)pb.mu, (const void*)pb.cond,
                        (const void*)pb.spk, (const void*)pb.out, (const void*)p->kv, (const void*)p->cnn})
    key = mix(key, reinterpret_cast<uint64_t>(q));
  if (nsrc) {  // the noise buffer and temperature are baked into the gather launch
    uint32_t tb = 0;
    std::memcpy(&tb, &nsrc->temperature, 4);
    key = mix(mix(mix(key, reinterpret_cast<uint64_t>(nsrc->noise)), (uint64_t)nsrc->frames), tb);
  }
  if (s->slot_seen.size() > 4096) s->slot_seen.clear();
  if ((flags & T2W_FLAG_GRAPH) && (s->graphs.count(key) || ++s->slot_seen[key] >= 2))
    return replay(s, key, st, [&](cudaStream_t cs) { return enqueue_solve(s, pl, pb, ws, cs, nullptr, p, nsrc); });
  T2W_TRY(enqueue_solve(s, pl, pb, ws, st, nullptr, p, nsrc));
  ++s->n_eager;
  return T2W_OK;
}

// The key lists, conv rows and noise columns of a window solve over library-kept caches (records already checked).
// fresh holds 2 * sum T new slots: request i's CFG row h takes T_i of them at fresh_off[h * n + i].
bool plan_cached(const t2w_config& c, const t2w_slots* p, int n, const int32_t* T, const uint8_t* keep,
                 const std::vector<CacheRecord*>& recs, const std::vector<int32_t>& fresh, Plan& pl) {
  std::vector<int> kv_len(2 * n), rd(2 * n), wr(2 * n);
  std::vector<int> kv_idx;
  size_t total = 0;
  for (int r = 0; r < 2 * n; ++r) total += recs[r % n]->keys[r / n].size() + (size_t)T[r % n];
  kv_idx.reserve(total);
  size_t fo = 0;
  std::vector<size_t> fresh_off(2 * n);
  for (int h = 0; h < 2; ++h)
    for (int i = 0; i < n; ++i) {
      fresh_off[h * n + i] = fo;
      fo += (size_t)T[i];
    }
  for (int r = 0; r < 2 * n; ++r) {
    const int i = r % n, h = r / n;
    const std::vector<int32_t>& k = recs[i]->keys[h];
    kv_idx.insert(kv_idx.end(), k.begin(), k.end());  // cached keys, then the window's new slots
    kv_idx.insert(kv_idx.end(), fresh.begin() + fresh_off[r], fresh.begin() + fresh_off[r] + T[i]);
    kv_len[r] = (int)k.size() + T[i];
    rd[r] = recs[i]->rowslot[h];
    wr[r] = keep[i] ? rd[r] : 0;  // row slot 0: scratch target of rows that keep nothing
  }
  if (!make_plan_slots(c, n, T, kv_len.data(), kv_idx.data(), rd.data(), wr.data(), p->n_slots, p->n_rowslots, pl))
    return false;
  pl.gather = true;
  pl.tok_col.clear();
  pl.tok_col.reserve(pl.n_tok);
  for (int i = 0; i < n; ++i)
    for (int t = 0; t < T[i]; ++t) pl.tok_col.push_back((int)recs[i]->keys[0].size() + t);
  return true;
}

// Records of a cached batch: every handle live and used once, every window inside the noise.
int cached_records(t2w_slots* p, const t2w_cached_batch* b, std::vector<CacheRecord*>& recs, long long* new_slots) {
  const int n = b->n_streams;
  if (n <= 0 || !b->handle || !b->chunk_len || !b->keep || b->noise_frames <= 0) return T2W_ERR_INVALID;
  std::vector<int32_t> ids(b->handle, b->handle + n);
  std::sort(ids.begin(), ids.end());
  if (std::adjacent_find(ids.begin(), ids.end()) != ids.end()) return T2W_ERR_INVALID;
  recs.resize(n);
  long long need = 0;
  for (int i = 0; i < n; ++i) {
    recs[i] = p->reg.find(b->handle[i]);
    if (!recs[i] || b->chunk_len[i] <= 0) return T2W_ERR_INVALID;
    if ((long long)recs[i]->keys[0].size() + b->chunk_len[i] > b->noise_frames) return T2W_ERR_INVALID;
    need += 2ll * b->chunk_len[i];
  }
  *new_slots = need;
  return T2W_OK;
}

}  // namespace

extern "C" {

int t2w_version(void) { return 1; }

int t2w_last_cuda_error(void) { return g_last_cuda_error; }

int t2w_device_ok(int device) {
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return 0;
  return p.major == 10 ? 1 : 0;
}

int t2w_create(const t2w_config* cfg, const float* t_sched, const float* const* weights, int32_t n_weights,
               int32_t precision, void* stream, t2w_solver** out) {
  if (!cfg || !weights || !out || !valid_cfg(*cfg)) return T2W_ERR_INVALID;
  const t2w_config& c = *cfg;
  const bool fp8 = precision == T2W_PREC_FP8;
  if (precision != T2W_PREC_BF16 && !fp8) return T2W_ERR_INVALID;
  // the FP8 GEMM tiles N by 256 and K by 128
  if (fp8 && (c.hidden % 256 || c.ffn % 256 || c.hidden % 128)) return T2W_ERR_UNSUPPORTED;
  if (n_weights != T2W_W_COUNT + c.depth * T2W_B_COUNT) return T2W_ERR_INVALID;
  for (int i = 0; i < n_weights; ++i)
    if (!weights[i]) return T2W_ERR_INVALID;
  int dev = 0;
  T2W_CUDA(cudaGetDevice(&dev));
  if (!t2w_device_ok(dev)) return T2W_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = c.hidden, F = c.ffn, mel = c.mel, S = c.steps;

  // arena: bf16 matrices, then fp32 vectors and tables
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_in = take((size_t)H * 4 * mel * 2), o_fin = take((size_t)mel * H * 2);
  const size_t o_bin = take(H * 4), o_bfin = take(mel * 4);
  const size_t o_mods = take((size_t)S * c.depth * 9 * H * 4), o_fmods = take((size_t)S * 2 * H * 4);
  const size_t o_dts = take(S * 4), o_ts = take(S * 4), o_freq = take(c.freq_dim * 4), o_st = take((size_t)S * H * 4);
  const size_t o_err = take(16);
  // per block: the six matrices (bf16, or e4m3 plus per-1x128-block scale atoms), then the vectors
  const size_t eb = fp8 ? 1 : 2;
  const int mat_n[6] = {3 * H, H, H, H, F, H}, mat_k[6] = {H, H, 3 * H, 3 * H, H, F};
  std::vector<size_t> ob(c.depth * 24);
  for (int b = 0; b < c.depth; ++b) {
    size_t* q = &ob[b * 24];
    for (int i = 0; i < 6; ++i) q[i] = take((size_t)mat_n[i] * mat_k[i] * eb);
    for (int i = 0; i < 6; ++i) q[18 + i] = take(fp8 ? gemm8_sf_bytes(mat_n[i], mat_k[i]) : 0);
    q[6] = take(3 * H * 4);
    q[7] = take(c.head_dim * 4);
    q[8] = take(c.head_dim * 4);
    q[9] = take(c.head_dim * 4);
    q[10] = take(c.head_dim * 4);
    q[11] = take(H * 4);
    q[12] = take(H * 4);
    q[13] = take(H * 4);
    q[14] = take(H * 4);
    q[15] = take(H * 4);
    q[16] = take(F * 4);
    q[17] = take(H * 4);
  }
  t2w_solver* s = new t2w_solver();
  s->cfg = c;
  s->precision = precision;
  s->device = dev;
  if (cudaMalloc(&s->arena, off) != cudaSuccess) {
    delete s;
    return T2W_ERR_OOM;
  }
  void* A = s->arena;
  auto fail = [&](int rc) {
    cudaFree(s->arena);
    delete s;
    return rc;
  };
  auto W = [&](int slot) { return weights[slot]; };
  auto BWp = [&](int b, int slot) { return weights[T2W_W_COUNT + b * T2W_B_COUNT + slot]; };
  auto copyv = [&](float* dst, const float* src, size_t n) {
    return cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess;
  };
  s->w_in = at<__nv_bfloat16>(A, o_in);
  s->w_fin = at<__nv_bfloat16>(A, o_fin);
  s->b_in = at<float>(A, o_bin);
  s->b_fin = at<float>(A, o_bfin);
  s->mods = at<float>(A, o_mods);
  s->final_mods = at<float>(A, o_fmods);
  s->dts_dev = at<float>(A, o_dts);
  s->err = at<int>(A, o_err);
  if (launch_f32_to_bf16(W(T2W_W_IN_W), s->w_in, (long long)H * 4 * mel, st) ||
      launch_f32_to_bf16(W(T2W_W_FINAL_W), s->w_fin, (long long)mel * H, st) || !copyv(s->b_in, W(T2W_W_IN_B), H) ||
      !copyv(s->b_fin, W(T2W_W_FINAL_B), mel))
    return fail(T2W_ERR_CUDA);
  s->blk.resize(c.depth);
  std::vector<const float*> ada_w(c.depth), ada_b(c.depth);
  // FP8: fp32 staging of one weight matrix in the layout that is quantised ([N, Kt], conv taps tap-major)
  float* tmp = nullptr;
  if (fp8 && cudaMalloc(reinterpret_cast<void**>(&tmp), (size_t)std::max(3 * H * H, F * H) * 4) != cudaSuccess)
    return fail(T2W_ERR_OOM);
  auto fail2 = [&](int rc) {
    if (tmp) cudaFree(tmp);
    return fail(rc);
  };
  for (int b = 0; b < c.depth; ++b) {
    BlockW& w = s->blk[b];
    const size_t* q = &ob[b * 24];
    w.b_qkv = at<float>(A, q[6]);
    w.qn_w = at<float>(A, q[7]);
    w.qn_b = at<float>(A, q[8]);
    w.kn_w = at<float>(A, q[9]);
    w.kn_b = at<float>(A, q[10]);
    w.b_proj = at<float>(A, q[11]);
    w.b_c1 = at<float>(A, q[12]);
    w.cln_w = at<float>(A, q[13]);
    w.cln_b = at<float>(A, q[14]);
    w.b_c2 = at<float>(A, q[15]);
    w.b_fc1 = at<float>(A, q[16]);
    w.b_fc2 = at<float>(A, q[17]);
    const long long HH = (long long)H * H;
    bool ok = copyv(w.b_qkv, BWp(b, T2W_B_Q_B), H) && copyv(w.b_qkv + H, BWp(b, T2W_B_K_B), H) &&
              copyv(w.b_qkv + 2 * H, BWp(b, T2W_B_V_B), H) && copyv(w.qn_w, BWp(b, T2W_B_QN_W), c.head_dim) &&
              copyv(w.qn_b, BWp(b, T2W_B_QN_B), c.head_dim) && copyv(w.kn_w, BWp(b, T2W_B_KN_W), c.head_dim) &&
              copyv(w.kn_b, BWp(b, T2W_B_KN_B), c.head_dim) && copyv(w.b_proj, BWp(b, T2W_B_PROJ_B), H) &&
              copyv(w.b_c1, BWp(b, T2W_B_C1_B), H) && copyv(w.cln_w, BWp(b, T2W_B_CLN_W), H) &&
              copyv(w.cln_b, BWp(b, T2W_B_CLN_B), H) && copyv(w.b_c2, BWp(b, T2W_B_C2_B), H) &&
              copyv(w.b_fc1, BWp(b, T2W_B_FC1_B), F) && copyv(w.b_fc2, BWp(b, T2W_B_FC2_B), H);
    if (!ok) return fail2(T2W_ERR_CUDA);
    if (fp8) {
      for (int i = 0; i < 6; ++i) {
        w.w8[i] = at<uint8_t>(A, q[i]);
        w.sf8[i] = at<uint8_t>(A, q[18 + i]);
      }
      ok = copyv(tmp, BWp(b, T2W_B_Q_W), HH) && copyv(tmp + HH, BWp(b, T2W_B_K_W), HH) &&
           copyv(tmp + 2 * HH, BWp(b, T2W_B_V_W), HH) &&
           !launch_quant_weight(tmp, 3 * H, H, w.w8[W8_QKV], w.sf8[W8_QKV], st) &&
           !launch_quant_weight(BWp(b, T2W_B_PROJ_W), H, H, w.w8[W8_PROJ], w.sf8[W8_PROJ], st) &&
           !launch_conv_weight_f32(BWp(b, T2W_B_C1_W), tmp, H, H, 3, st) &&
           !launch_quant_weight(tmp, H, 3 * H, w.w8[W8_C1], w.sf8[W8_C1], st) &&
           !launch_conv_weight_f32(BWp(b, T2W_B_C2_W), tmp, H, H, 3, st) &&
           !launch_quant_weight(tmp, H, 3 * H, w.w8[W8_C2], w.sf8[W8_C2], st) &&
           !launch_quant_weight(BWp(b, T2W_B_FC1_W), F, H, w.w8[W8_FC1], w.sf8[W8_FC1], st) &&
           !launch_quant_weight(BWp(b, T2W_B_FC2_W), H, F, w.w8[W8_FC2], w.sf8[W8_FC2], st);
      if (!ok) return fail2(T2W_ERR_CUDA);
      for (int i = 0; i < 6; ++i)
        if (!make_tmap_2d(&w.t8[i], w.w8[i], 1, mat_n[i], mat_k[i], mat_k[i], 256, 128)) return fail2(T2W_ERR_INVALID);
    } else {
      w.qkv = at<__nv_bfloat16>(A, q[0]);
      w.proj = at<__nv_bfloat16>(A, q[1]);
      w.c1 = at<__nv_bfloat16>(A, q[2]);
      w.c2 = at<__nv_bfloat16>(A, q[3]);
      w.fc1 = at<__nv_bfloat16>(A, q[4]);
      w.fc2 = at<__nv_bfloat16>(A, q[5]);
      ok = !launch_f32_to_bf16(BWp(b, T2W_B_Q_W), w.qkv, HH, st) &&
           !launch_f32_to_bf16(BWp(b, T2W_B_K_W), w.qkv + HH, HH, st) &&
           !launch_f32_to_bf16(BWp(b, T2W_B_V_W), w.qkv + 2 * HH, HH, st) &&
           !launch_f32_to_bf16(BWp(b, T2W_B_PROJ_W), w.proj, HH, st) &&
           !launch_conv_weight(BWp(b, T2W_B_C1_W), w.c1, H, H, 3, st) &&
           !launch_conv_weight(BWp(b, T2W_B_C2_W), w.c2, H, H, 3, st) &&
           !launch_f32_to_bf16(BWp(b, T2W_B_FC1_W), w.fc1, (long long)F * H, st) &&
           !launch_f32_to_bf16(BWp(b, T2W_B_FC2_W), w.fc2, (long long)H * F, st);
      if (!ok) return fail2(T2W_ERR_CUDA);
      if (!weight_map(&w.tm_qkv, w.qkv, 3 * H, H) || !weight_map(&w.tm_proj, w.proj, H, H) ||
          !weight_map(&w.tm_c1, w.c1, H, 3 * H) || !weight_map(&w.tm_c2, w.c2, H, 3 * H) ||
          !weight_map(&w.tm_fc1, w.fc1, F, H) || !weight_map(&w.tm_fc2, w.fc2, H, F))
        return fail2(T2W_ERR_INVALID);
    }
    ada_w[b] = BWp(b, T2W_B_ADA_W);
    ada_b[b] = BWp(b, T2W_B_ADA_B);
  }
  if (!weight_map(&s->tm_in, s->w_in, H, 4 * mel) || !weight_map(&s->tm_fin, s->w_fin, mel, H)) return fail2(T2W_ERR_INVALID);

  // t schedule: the caller's fp32 (t, dt) pairs, else the cosine schedule in double rounded to fp32
  std::vector<float> ts(S);
  s->dts.resize(S);
  if (t_sched) {
    for (int i = 0; i < S; ++i) {
      ts[i] = t_sched[2 * i];
      s->dts[i] = t_sched[2 * i + 1];
    }
  } else {
    std::vector<double> span(S + 1);
    for (int i = 0; i <= S; ++i) span[i] = 1.0 - std::cos((double)i / S * 0.5 * M_PI);
    double t = span[0];
    for (int i = 0; i < S; ++i) {
      ts[i] = (float)t;
      s->dts[i] = (float)(span[i + 1] - t);
      t += span[i + 1] - t;
    }
  }
  const int half = c.freq_dim / 2;
  std::vector<float> freqs(half);
  const float lnp = (float)(-std::log((double)c.max_period));
  for (int k = 0; k < half; ++k) freqs[k] = std::exp(lnp * (float)k / (float)half);
  float* ts_dev = at<float>(A, o_ts);
  float* fr_dev = at<float>(A, o_freq);
  if (cudaMemcpyAsync(ts_dev, ts.data(), S * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(s->dts_dev, s->dts.data(), S * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(fr_dev, freqs.data(), half * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemsetAsync(s->err, 0, 16, st) != cudaSuccess)
    return fail2(T2W_ERR_CUDA);
  const int rc = launch_temb_mods(ts_dev, S, fr_dev, c.freq_dim, c.t_scale, W(T2W_W_TEMB_FC1_W), W(T2W_W_TEMB_FC1_B),
                                  W(T2W_W_TEMB_FC2_W), W(T2W_W_TEMB_FC2_B), H, ada_w.data(), ada_b.data(), c.depth,
                                  W(T2W_W_FINAL_ADA_W), W(T2W_W_FINAL_ADA_B), at<float>(A, o_st), s->mods,
                                  s->final_mods, st);
  if (rc) return fail2(rc);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return fail2(T2W_ERR_CUDA);
  }
  if (tmp) cudaFree(tmp);
  *out = s;
  return T2W_OK;
}

int t2w_destroy(t2w_solver* s) {
  if (!s) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  for (auto& kv : s->graphs) {
    cudaGraphExecDestroy(kv.second.exec);
    cudaEventDestroy(kv.second.done);
  }
  if (s->cap_stream) cudaStreamDestroy(s->cap_stream);
  for (cudaEvent_t e : s->prof_events) cudaEventDestroy(e);
  for (auto& sg : s->staging) {
    if (sg.done) {
      cudaEventSynchronize(sg.done);
      cudaEventDestroy(sg.done);
    }
    if (sg.host) cudaFreeHost(sg.host);
  }
  cudaFree(s->arena);
  delete s;
  return T2W_OK;
}

size_t t2w_workspace_bytes(const t2w_solver* s, int32_t n, const int32_t* P, const int32_t* T) {
  if (!s) return 0;
  Plan pl;
  if (!make_plan(s->cfg, n, P, T, pl)) return 0;
  return layout(s->cfg, pl, s->precision == T2W_PREC_FP8).total;
}

int t2w_solve_packed(t2w_solver* s, const t2w_batch* b, void* ws, size_t ws_bytes, uint32_t flags, void* stream) {
  if (!s || !b || !ws || !b->x0 || !b->mu || !b->cond || !b->spk || !b->out) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  Plan pl;
  if (!make_plan(s->cfg, b->n_streams, b->prompt_len, b->chunk_len, pl)) return T2W_ERR_INVALID;
  if (layout(s->cfg, pl, s->precision == T2W_PREC_FP8).total > ws_bytes) return T2W_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) & 255) return T2W_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uintptr_t wkey = reinterpret_cast<uintptr_t>(ws);
  auto it = s->ws_meta.find(wkey);
  if (it == s->ws_meta.end() || it->second != pl.key) T2W_TRY(upload_meta(s, pl, ws, st));
  if (!(flags & T2W_FLAG_GRAPH)) {
    T2W_TRY(enqueue_solve(s, pl, *b, ws, st));
    ++s->n_eager;
    return T2W_OK;
  }
  uint64_t key = pl.key;
  for (const void* p : {(const void*)ws, (const void*)b->x0, (const void*)b->mu, (const void*)b->cond,
                        (const void*)b->spk, (const void*)b->out})
    key = mix(key, reinterpret_cast<uint64_t>(p));
  return replay(s, key, st, [&](cudaStream_t cs) { return enqueue_solve(s, pl, *b, ws, cs); });
}

int t2w_profile_solve(t2w_solver* s, const t2w_batch* b, void* ws, size_t ws_bytes, void* stream, float* ms,
                      int32_t* launches) {
  if (!s || !b || !ws || !ms || !launches || !b->x0 || !b->mu || !b->cond || !b->spk || !b->out) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  Plan pl;
  if (!make_plan(s->cfg, b->n_streams, b->prompt_len, b->chunk_len, pl)) return T2W_ERR_INVALID;
  if (layout(s->cfg, pl, s->precision == T2W_PREC_FP8).total > ws_bytes || (reinterpret_cast<uintptr_t>(ws) & 255))
    return T2W_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto it = s->ws_meta.find(reinterpret_cast<uintptr_t>(ws));
  if (it == s->ws_meta.end() || it->second != pl.key) T2W_TRY(upload_meta(s, pl, ws, st));
  Prof prof;
  prof.events = &s->prof_events;
  T2W_TRY(enqueue_solve(s, pl, *b, ws, st, &prof));
  T2W_CUDA(cudaStreamSynchronize(st));
  for (int c = 0; c < T2W_KC_COUNT; ++c) {
    ms[c] = 0.f;
    launches[c] = 0;
  }
  for (size_t i = 0; i + 1 < prof.cls.size(); ++i) {
    float t = 0.f;
    T2W_CUDA(cudaEventElapsedTime(&t, s->prof_events[i], s->prof_events[i + 1]));
    const int c = prof.cls[i];
    if (c >= 0 && c < T2W_KC_COUNT) {
      ms[c] += t;
      launches[c] += 1;
    }
  }
  ++s->n_eager;
  return T2W_OK;
}

int t2w_test_wait_timeout(t2w_solver* s, int64_t limit_ns, void* stream) {
  if (!s || limit_ns < 100000 || limit_ns > (int64_t)kWaitLimitNs) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 256 rows of the solver's width: one block counter that nothing publishes (zero), fp32 h, bf16 out
  const int rows = 256, C = s->cfg.hidden;
  const size_t hb = (size_t)rows * C * 4, ob = (size_t)rows * C * 2, fb = 256;
  uint8_t* buf = nullptr;
  T2W_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&buf), hb + ob + fb, st));
  int rc = T2W_OK;
  cudaError_t e = cudaMemsetAsync(buf, 0, hb + ob + fb, st);
  if (e == cudaSuccess) {
    RowWait w;
    w.flags = reinterpret_cast<const int*>(buf + hb + ob);
    w.target = 1;  // never reached: every warp gives up after limit_ns and records T2W_ERR_TIMEOUT
    w.err = s->err;
    w.limit_ns = (unsigned long long)limit_ns;
    const float* v = s->final_mods;  // any finite [H] vectors serve as shift and scale
    rc = launch_add_ln_mod(reinterpret_cast<float*>(buf), nullptr, nullptr, v, v + C, s->cfg.eps_final, rows, C,
                           row_out_bf16(reinterpret_cast<__nv_bfloat16*>(buf + hb)), nullptr, st, w);
  } else {
    set_cuda_error(e);
    rc = T2W_ERR_CUDA;
  }
  cudaFreeAsync(buf, st);
  return rc;
}

int t2w_check(t2w_solver* s) {
  if (!s) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  int v = 0;
  T2W_CUDA(cudaMemcpy(&v, s->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) {
    T2W_CUDA(cudaMemset(s->err, 0, sizeof(int)));
    return v;
  }
  return T2W_OK;
}

int t2w_mods(const t2w_solver* s, float* mods, float* final_mods, float* dts, void* stream) {
  if (!s) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  const t2w_config& c = s->cfg;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mods) T2W_CUDA(cudaMemcpyAsync(mods, s->mods, (size_t)c.steps * c.depth * 9 * c.hidden * 4, cudaMemcpyDeviceToDevice, st));
  if (final_mods)
    T2W_CUDA(cudaMemcpyAsync(final_mods, s->final_mods, (size_t)c.steps * 2 * c.hidden * 4, cudaMemcpyDeviceToDevice, st));
  if (dts) T2W_CUDA(cudaMemcpyAsync(dts, s->dts_dev, (size_t)c.steps * 4, cudaMemcpyDeviceToDevice, st));
  return T2W_OK;
}

int t2w_counts(const t2w_solver* s, int64_t* replays, int64_t* captures, int64_t* eager) {
  if (!s) return T2W_ERR_INVALID;
  if (replays) *replays = s->n_replays;
  if (captures) *captures = s->n_captures;
  if (eager) *eager = s->n_eager;
  return T2W_OK;
}

int t2w_slots_create(const t2w_solver* s, int32_t n_slots, int32_t n_rowslots, t2w_slots** out) {
  if (!s || !out || n_slots <= 0 || n_rowslots <= 0) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  t2w_slots* p = new t2w_slots();
  p->device = s->device;
  p->n_slots = n_slots;
  p->n_rowslots = n_rowslots;
  p->n_sb = s->cfg.steps * s->cfg.depth;
  p->H = s->cfg.hidden;
  p->reg.init(n_slots, n_rowslots);
  const size_t kv_bytes = (size_t)p->n_sb * p->kv_sb() * 2, cnn_bytes = (size_t)p->n_sb * p->cnn_sb() * 2;
  if (cudaMalloc(reinterpret_cast<void**>(&p->kv), kv_bytes) != cudaSuccess) {
    delete p;
    return T2W_ERR_OOM;
  }
  if (cudaMalloc(reinterpret_cast<void**>(&p->cnn), cnn_bytes) != cudaSuccess) {
    cudaFree(p->kv);
    delete p;
    return T2W_ERR_OOM;
  }
  // finite contents everywhere (slots are read only through key lists, but a zero pool keeps stray reads harmless)
  if (cudaMemset(p->kv, 0, kv_bytes) != cudaSuccess || cudaMemset(p->cnn, 0, cnn_bytes) != cudaSuccess) {
    cudaFree(p->kv);
    cudaFree(p->cnn);
    delete p;
    return T2W_ERR_CUDA;
  }
  *out = p;
  return T2W_OK;
}

int t2w_slots_destroy(t2w_slots* p) {
  if (!p) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(p->device);
  cudaFree(p->kv);
  cudaFree(p->cnn);
  delete p;
  return T2W_OK;
}

int t2w_slots_copy(t2w_slots* p, const int32_t* src, const int32_t* dst, int32_t n, void* stream) {
  if (!p || n < 0 || (n > 0 && (!src || !dst))) return T2W_ERR_INVALID;
  if (n == 0) return T2W_OK;
  T2W_ON_DEVICE(p->device);
  for (int i = 0; i < n; ++i)
    if (src[i] < 0 || src[i] >= p->n_slots || dst[i] < 0 || dst[i] >= p->n_slots) return T2W_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* d = nullptr;
  T2W_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d), 2 * (size_t)n * 4, st));
  T2W_CUDA(cudaMemcpyAsync(d, src, (size_t)n * 4, cudaMemcpyHostToDevice, st));
  T2W_CUDA(cudaMemcpyAsync(d + n, dst, (size_t)n * 4, cudaMemcpyHostToDevice, st));
  const int rc = launch_slot_copy(p->kv, 2 * p->H, p->kv_sb(), p->n_sb, d, d + n, n, st);
  cudaFreeAsync(d, st);
  return rc;
}

int t2w_slots_copy_row(t2w_slots* p, int32_t src, int32_t dst, void* stream) {
  if (!p || src >= p->n_rowslots || dst < 0 || dst >= p->n_rowslots) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(p->device);
  return launch_rowslot_copy(p->cnn, p->cnn_slot(), p->cnn_sb(), p->n_sb, src < 0 ? -1 : src, dst,
                             static_cast<cudaStream_t>(stream));
}

int t2w_slots_pools(const t2w_slots* p, void** kv, void** cnn, int32_t* n_sb, int32_t* n_slots, int32_t* n_rowslots,
                    int32_t* hidden) {
  if (!p || !kv || !cnn || !n_sb || !n_slots || !n_rowslots || !hidden) return T2W_ERR_INVALID;
  *kv = p->kv;
  *cnn = p->cnn;
  *n_sb = p->n_sb;
  *n_slots = p->n_slots;
  *n_rowslots = p->n_rowslots;
  *hidden = p->H;
  return T2W_OK;
}

size_t t2w_slot_workspace_bytes(const t2w_solver* s, const t2w_slots* p, const t2w_slot_batch* b) {
  if (!s || !p || !b) return 0;
  Plan pl;
  if (!make_plan_slots(s->cfg, b->n_streams, b->chunk_len, b->kv_len, b->kv_idx, b->cnn_rd, b->cnn_wr, p->n_slots,
                       p->n_rowslots, pl))
    return 0;
  return layout(s->cfg, pl, false).total;
}

int t2w_solve_slots(t2w_solver* s, t2w_slots* p, const t2w_slot_batch* b, void* ws, size_t ws_bytes, uint32_t flags,
                    void* stream) {
  if (!s || !p || !b || !ws || !b->x0 || !b->mu || !b->spk || !b->out) return T2W_ERR_INVALID;
  if (s->precision != T2W_PREC_BF16) return T2W_ERR_UNSUPPORTED;
  if (p->device != s->device) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  Plan pl;
  if (!make_plan_slots(s->cfg, b->n_streams, b->chunk_len, b->kv_len, b->kv_idx, b->cnn_rd, b->cnn_wr, p->n_slots,
                       p->n_rowslots, pl))
    return T2W_ERR_INVALID;
  if (layout(s->cfg, pl, false).total > ws_bytes) return T2W_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) & 255) return T2W_ERR_INVALID;
  // the window solve is the packed solve's body with P = 0 rows: every row a window
  t2w_batch pb{};
  pb.n_streams = b->n_streams;
  pb.x0 = b->x0;
  pb.mu = b->mu;
  pb.cond = b->cond;
  pb.spk = b->spk;
  pb.out = b->out;
  return run_slot_plan(s, p, pl, pb, ws, flags, static_cast<cudaStream_t>(stream), nullptr);
}

// ---- caches kept by the library -----------------------------------------------------------------------------------

int t2w_cache_new(t2w_slots* p, int32_t keep, void* stream, int32_t* handle) {
  if (!p || !handle) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(p->device);
  std::lock_guard<std::mutex> lock(p->mu);
  const int32_t id = p->reg.open();
  if (id < 0) return T2W_ERR_EXHAUSTED;
  CacheRecord* r = p->reg.find(id);
  r->keep = keep;
  for (int h = 0; h < 2; ++h) {
    const int rc = launch_rowslot_copy(p->cnn, p->cnn_slot(), p->cnn_sb(), p->n_sb, -1, r->rowslot[h],
                                       static_cast<cudaStream_t>(stream));
    if (rc) {
      p->reg.close(id);
      return rc;
    }
  }
  *handle = id;
  return T2W_OK;
}

int t2w_cache_release(t2w_slots* p, int32_t handle) {
  if (!p) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lock(p->mu);
  if (!p->reg.find(handle)) return T2W_ERR_INVALID;
  p->reg.close(handle);
  return T2W_OK;
}

int t2w_cache_clone(t2w_slots* p, int32_t handle, void* stream, int32_t* out) {
  if (!p || !out) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(p->device);
  std::lock_guard<std::mutex> lock(p->mu);
  if (!p->reg.find(handle)) return T2W_ERR_INVALID;
  const int32_t id = p->reg.open();  // may grow the record table: look both records up afterwards
  if (id < 0) return T2W_ERR_EXHAUSTED;
  CacheRecord* src = p->reg.find(handle);
  CacheRecord* dst = p->reg.find(id);
  dst->keep = src->keep;
  const int n = (int)src->keys[0].size();
  std::vector<int32_t> ids(2 * (size_t)n);
  if (!p->reg.slots.take(2 * n, ids.data())) {
    p->reg.close(id);
    return T2W_ERR_EXHAUSTED;
  }
  dst->keys[0].assign(ids.begin(), ids.begin() + n);
  dst->keys[1].assign(ids.begin() + n, ids.end());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = T2W_OK;
  for (int h = 0; h < 2 && !rc; ++h)
    rc = launch_rowslot_copy(p->cnn, p->cnn_slot(), p->cnn_sb(), p->n_sb, src->rowslot[h], dst->rowslot[h], st);
  if (!rc && n > 0) {
    std::vector<int32_t> from(src->keys[0]);
    from.insert(from.end(), src->keys[1].begin(), src->keys[1].end());
    int* d = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d), 4 * (size_t)n * 4, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d, from.data(), 2 * (size_t)n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d + 2 * n, ids.data(), 2 * (size_t)n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) rc = launch_slot_copy(p->kv, 2 * p->H, p->kv_sb(), p->n_sb, d, d + 2 * n, 2 * n, st);
    if (d) cudaFreeAsync(d, st);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      rc = T2W_ERR_CUDA;
    }
    // the host index vectors above are pageable: the copies complete before cudaMemcpyAsync returns
  }
  if (rc) {
    p->reg.close(id);
    return rc;
  }
  *out = id;
  return T2W_OK;
}

int t2w_cache_get(const t2w_slots* p, int32_t handle, t2w_cache_info* info) {
  if (!p || !info) return T2W_ERR_INVALID;
  t2w_slots* q = const_cast<t2w_slots*>(p);
  std::lock_guard<std::mutex> lock(q->mu);
  const CacheRecord* r = q->reg.find(handle);
  if (!r) return T2W_ERR_INVALID;
  info->length = (int32_t)r->keys[0].size();
  info->keep = r->keep;
  info->rowslot[0] = r->rowslot[0];
  info->rowslot[1] = r->rowslot[1];
  return T2W_OK;
}

int t2w_cache_set_keep(t2w_slots* p, int32_t handle, int32_t keep) {
  if (!p) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lock(p->mu);
  CacheRecord* r = p->reg.find(handle);
  if (!r) return T2W_ERR_INVALID;
  r->keep = keep;
  return T2W_OK;
}

int t2w_cache_keys(const t2w_slots* p, int32_t handle, int32_t half, int32_t* slots, int32_t cap) {
  if (!p || (half != 0 && half != 1) || cap < 0 || (cap > 0 && !slots)) return T2W_ERR_INVALID;
  t2w_slots* q = const_cast<t2w_slots*>(p);
  std::lock_guard<std::mutex> lock(q->mu);
  const CacheRecord* r = q->reg.find(handle);
  if (!r || (size_t)cap < r->keys[half].size()) return T2W_ERR_INVALID;
  std::copy(r->keys[half].begin(), r->keys[half].end(), slots);
  return T2W_OK;
}

int t2w_cache_reserve(t2w_slots* p, int32_t handle, int32_t n, int32_t* slots) {
  if (!p || n < 0 || (n > 0 && !slots)) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lock(p->mu);
  CacheRecord* r = p->reg.find(handle);
  if (!r || !r->keys[0].empty() || !r->keys[1].empty()) return T2W_ERR_INVALID;
  if (n == 0) return T2W_OK;
  if (!p->reg.slots.take(2 * n, slots)) return T2W_ERR_EXHAUSTED;
  r->keys[0].assign(slots, slots + n);
  r->keys[1].assign(slots + n, slots + 2 * n);
  return T2W_OK;
}

int t2w_slots_usage(const t2w_slots* p, int32_t* keys_in_use, int32_t* rowslots_free, int32_t* caches) {
  if (!p) return T2W_ERR_INVALID;
  t2w_slots* q = const_cast<t2w_slots*>(p);
  std::lock_guard<std::mutex> lock(q->mu);
  if (keys_in_use) *keys_in_use = q->reg.slots.used();
  if (rowslots_free) *rowslots_free = q->reg.rows.available();
  if (caches) *caches = q->reg.live();
  return T2W_OK;
}

size_t t2w_cached_workspace_bytes(const t2w_solver* s, const t2w_slots* p, const t2w_cached_batch* b) {
  if (!s || !p || !b) return 0;
  t2w_slots* q = const_cast<t2w_slots*>(p);
  std::lock_guard<std::mutex> lock(q->mu);
  std::vector<CacheRecord*> recs;
  long long need = 0;
  if (cached_records(q, b, recs, &need) != T2W_OK) return 0;
  std::vector<int32_t> fresh((size_t)need, 0);  // sizes only: slot 0 stands in for every new slot
  Plan pl;
  if (!plan_cached(s->cfg, q, b->n_streams, b->chunk_len, b->keep, recs, fresh, pl)) return 0;
  return layout(s->cfg, pl, false).total;
}

int t2w_solve_cached(t2w_solver* s, t2w_slots* p, const t2w_cached_batch* b, void* ws, size_t ws_bytes, uint32_t flags,
                     void* stream) {
  if (!s || !p || !b || !ws || !b->noise || !b->mu || !b->spk || !b->out) return T2W_ERR_INVALID;
  if (s->precision != T2W_PREC_BF16) return T2W_ERR_UNSUPPORTED;
  if (p->device != s->device) return T2W_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(ws) & 255) return T2W_ERR_INVALID;
  T2W_ON_DEVICE(s->device);
  std::lock_guard<std::mutex> lock(p->mu);
  std::vector<CacheRecord*> recs;
  long long need = 0;
  T2W_TRY(cached_records(p, b, recs, &need));
  if (need > p->reg.slots.available()) return T2W_ERR_EXHAUSTED;
  std::vector<int32_t> fresh((size_t)need);
  p->reg.slots.take((int)need, fresh.data());
  auto undo = [&](int rc) {
    p->reg.slots.give(fresh.data(), fresh.size());
    return rc;
  };
  const int n = b->n_streams;
  Plan pl;
  if (!plan_cached(s->cfg, p, n, b->chunk_len, b->keep, recs, fresh, pl)) return undo(T2W_ERR_INVALID);
  const WsLayout L = layout(s->cfg, pl, false);
  if (L.total > ws_bytes) return undo(T2W_ERR_WORKSPACE);
  t2w_batch pb{};
  pb.n_streams = n;
  pb.x0 = at<float>(ws, L.x0g);
  pb.mu = b->mu;
  pb.cond = b->cond;
  pb.spk = b->spk;
  pb.out = b->out;
  NoiseSrc ns;
  ns.noise = b->noise;
  ns.frames = b->noise_frames;
  ns.temperature = b->temperature;
  const int rc = run_slot_plan(s, p, pl, pb, ws, flags, static_cast<cudaStream_t>(stream), &ns);
  if (rc) return undo(rc);
  // the reference's order and trim (dit_fast.py:480-490); final flushes hand their window's slots straight back
  size_t fo = 0;
  for (int h = 0; h < 2; ++h)
    for (int i = 0; i < n; ++i) {
      const int T = b->chunk_len[i];
      if (b->keep[i])
        p->reg.commit_window(*recs[i], h, fresh.data() + fo, T);
      else
        p->reg.slots.give(fresh.data() + fo, (size_t)T);
      fo += (size_t)T;
    }
  return T2W_OK;
}

int t2w_ln_mod(const float* h, int32_t ld_h, const float* shift, const float* scale1, float eps, int32_t rows,
               int32_t C, void* out, int32_t ld_out, const uint8_t* pad, void* stream) {
  if (!h || !shift || !scale1 || !out) return T2W_ERR_INVALID;
  return launch_ln_mod(h, ld_h, shift, scale1, eps, rows, C, static_cast<__nv_bfloat16*>(out), ld_out, pad,
                       static_cast<cudaStream_t>(stream));
}

int t2w_add_ln_mod(float* h, const void* y, const float* g, const float* shift, const float* scale1, float eps, int32_t rows,
                   int32_t C, void* out, const uint8_t* pad, void* stream) {
  if (!h || !shift || !scale1 || !out) return T2W_ERR_INVALID;
  return launch_add_ln_mod(h, static_cast<const __nv_bfloat16*>(y), g, shift, scale1, eps, rows, C,
                           row_out_bf16(static_cast<__nv_bfloat16*>(out)), pad, static_cast<cudaStream_t>(stream));
}

int t2w_ln_mish(const void* x, const float* w, const float* b, float eps, int32_t rows, int32_t C, void* out,
                const uint8_t* pad, void* stream) {
  if (!x || !w || !b || !out) return T2W_ERR_INVALID;
  return launch_ln_mish(static_cast<const __nv_bfloat16*>(x), w, b, eps, rows, C,
                        row_out_bf16(static_cast<__nv_bfloat16*>(out)), pad, static_cast<cudaStream_t>(stream));
}

size_t t2w_e4m3_sf_bytes(int32_t rows, int32_t C) {
  if (rows <= 0 || C <= 0 || C % 128) return 0;
  return gemm8_sf_bytes(rows, C);
}

int t2w_quant_e4m3(const void* x, int32_t rows, int32_t C, void* out, uint8_t* sf, int32_t n_layouts, int64_t layout_bytes,
                   void* stream) {
  if (!x || !out || !sf) return T2W_ERR_INVALID;
  RowOut o;
  o.out = out;
  o.sf = sf;
  o.n_layouts = n_layouts;
  o.layout_bytes = layout_bytes;
  return launch_quant_rows(static_cast<const __nv_bfloat16*>(x), rows, C, o, static_cast<cudaStream_t>(stream));
}

int t2w_quant_weight_e4m3(const float* w, int32_t N, int32_t Kt, void* w8, uint8_t* sf, void* stream) {
  return launch_quant_weight(w, N, Kt, static_cast<uint8_t*>(w8), sf, static_cast<cudaStream_t>(stream));
}

int t2w_add_ln_mod_e4m3(float* h, const void* y, const float* g, const float* shift, const float* scale1, float eps,
                        int32_t rows, int32_t C, void* out, uint8_t* sf, int32_t n_layouts, int64_t layout_bytes,
                        const uint8_t* pad, void* stream) {
  if (!h || !shift || !scale1 || !out || !sf) return T2W_ERR_INVALID;
  RowOut o;
  o.out = out;
  o.sf = sf;
  o.n_layouts = n_layouts;
  o.layout_bytes = layout_bytes;
  return launch_add_ln_mod(h, static_cast<const __nv_bfloat16*>(y), g, shift, scale1, eps, rows, C, o, pad,
                           static_cast<cudaStream_t>(stream));
}

int t2w_ln_mish_e4m3(const void* x, const float* w, const float* b, float eps, int32_t rows, int32_t C, void* out,
                     uint8_t* sf, int32_t n_layouts, int64_t layout_bytes, const uint8_t* pad, void* stream) {
  if (!x || !w || !b || !out || !sf) return T2W_ERR_INVALID;
  RowOut o;
  o.out = out;
  o.sf = sf;
  o.n_layouts = n_layouts;
  o.layout_bytes = layout_bytes;
  return launch_ln_mish(static_cast<const __nv_bfloat16*>(x), w, b, eps, rows, C, o, pad,
                        static_cast<cudaStream_t>(stream));
}

int t2w_gemm_e4m3(const void* A8, int32_t lda, int32_t rows_a, const uint8_t* sfa, int32_t sfa_layouts,
                  int64_t sfa_layout_bytes, const void* W8, const uint8_t* sfw, const float* bias, int32_t M, int32_t N,
                  int32_t K, int32_t taps, int32_t tap_row0, int32_t epi, void* out, int32_t ldo, uint8_t* out_sf,
                  const float* const* qk, float qk_eps, void* stream) {
  Gemm8Args g;
  g.A8 = A8;
  g.lda = lda;
  g.rows_a = rows_a;
  g.sfa = sfa;
  g.sfa_layouts = sfa_layouts;
  g.sfa_layout = sfa_layout_bytes;
  g.W8 = W8;
  g.sfw = sfw;
  g.bias = bias;
  g.M = M;
  g.N = N;
  g.K = K;
  g.taps = taps;
  g.tap_row0 = tap_row0;
  g.epi = epi;
  g.out = out;
  g.ldo = ldo;
  g.out_sf = out_sf;
  if (qk) {
    g.qn_w = qk[0];
    g.qn_b = qk[1];
    g.kn_w = qk[2];
    g.kn_b = qk[3];
  }
  g.qk_eps = qk_eps;
  return launch_gemm8(g, static_cast<cudaStream_t>(stream));
}

int t2w_gemm(const void* A, int32_t lda, int32_t rows_a, const void* W, const float* bias, int32_t M, int32_t N,
             int32_t K, int32_t taps, int32_t tap_row0, int32_t epi, void* out, int32_t ldo, const float* const* qk,
             float qk_eps, void* stream) {
  GemmArgs g;
  g.A = A;
  g.lda = lda;
  g.rows_a = rows_a;
  g.W = W;
  g.bias = bias;
  g.M = M;
  g.N = N;
  g.K = K;
  g.taps = taps;
  g.tap_row0 = tap_row0;
  g.epi = epi;
  g.out = out;
  g.ldo = ldo;
  if (qk && epi == T2W_EPI_QKV) {
    g.qn_w = qk[0];
    g.qn_b = qk[1];
    g.kn_w = qk[2];
    g.kn_b = qk[3];
  }
  if (qk && epi == T2W_EPI_RESID) g.gate = qk[0];
  g.qk_eps = qk_eps;
  return launch_gemm(g, static_cast<cudaStream_t>(stream));
}

int t2w_attn_varlen(const void* qkv, int32_t rows, int32_t heads, int32_t n_seq, const int32_t* seq_row,
                    const int32_t* seq_len, const int32_t* prompt_len, void* out, void* stream) {
  return attn_varlen_alloc(qkv, rows, heads, n_seq, seq_row, seq_len, prompt_len, out, nullptr, stream);
}

int t2w_attn_varlen_e4m3(const void* qkv, int32_t rows, int32_t heads, int32_t n_seq, const int32_t* seq_row,
                         const int32_t* seq_len, const int32_t* prompt_len, void* out, uint8_t* sf, void* stream) {
  if (!sf) return T2W_ERR_INVALID;
  return attn_varlen_alloc(qkv, rows, heads, n_seq, seq_row, seq_len, prompt_len, out, sf, stream);
}

int t2w_euler_cfg(float* x, const float* dphi, int32_t ld_dphi, const int32_t* tok_row, int32_t n_tok, int32_t mel,
                  int32_t half_rows, float dt, float w, void* hx, int32_t ld_hx, float* out, void* stream) {
  if (!x || !dphi || !tok_row) return T2W_ERR_INVALID;
  return launch_euler(x, dphi, ld_dphi, tok_row, n_tok, mel, half_rows, dt, w, static_cast<__nv_bfloat16*>(hx), ld_hx,
                      out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
