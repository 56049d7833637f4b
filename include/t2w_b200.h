/* C ABI of the B200 Token2Wav DiT/CFM solver (libt2w_b200.so).
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*); every entry point returns an int status (T2W_OK == 0,
 * negative on error) and never aborts the process.  Device pointers are CUDA global memory on the current device.
 * The solver enqueues all work on the given stream and does not synchronise unless a function says so.
 *
 * Reference interfaces replaced (paths inside InferMatrixLab/minicpm-o-4.5-single-gpu-engine):
 *   t2w_create            FastDiT.__init__            engine/runtime/dit_fast.py:100-155 (weights cast once, adaLN
 *                                                      modulations precomputed per step: dit_fast.py:157-178)
 *   t2w_solve_packed      FastDiT.solve               engine/runtime/dit_fast.py:432-495, and
 *                         BatchedToken2Wav._solve     engine/runtime/token2wav_batch.py:632-702 (CFG Euler solve)
 *   t2w_mods              FastDiT._modulations        engine/runtime/dit_fast.py:157-178
 *   t2w_ln_mod            ln_mod                      engine/runtime/dit_kernels.py:13-32
 *   t2w_add_ln_mod        add_ln_mod                  engine/runtime/dit_kernels.py:35-60
 *   t2w_ln_mish           ln_mish                     engine/runtime/dit_kernels.py:145-164
 *   t2w_gemm              F.linear calls of the block engine/runtime/dit_fast.py:283-301 (cuBLAS in the reference)
 *   t2w_attn_varlen       BatchPrefillWithPagedKVCacheWrapper.run  engine/runtime/dit_fast.py:291,347-367
 *   t2w_euler_cfg         the CFG combine + Euler step engine/runtime/dit_fast.py:302 / token2wav_batch.py:689-690
 */
#ifndef T2W_B200_H_
#define T2W_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define T2W_API __attribute__((visibility("default")))
#else
#define T2W_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define T2W_OK 0
#define T2W_ERR_INVALID (-1)     /* bad argument or shape */
#define T2W_ERR_CUDA (-2)        /* a CUDA runtime call failed (t2w_last_cuda_error gives the code) */
#define T2W_ERR_OOM (-3)         /* device allocation failed */
#define T2W_ERR_TIMEOUT (-4)     /* a kernel's bounded wait gave up (reported by t2w_check) */
#define T2W_ERR_UNSUPPORTED (-5) /* config outside the kernels' shape set, or no sm_100 device */
#define T2W_ERR_WORKSPACE (-6)   /* workspace too small */
#define T2W_ERR_EXHAUSTED (-7)   /* the slot pool, the conv-cache row slots or the cache handles are used up */

#define T2W_PREC_BF16 0 /* bf16 weights and activations, fp32 accumulate */
#define T2W_PREC_FP8 1  /* e4m3 weights (power-of-two scale per 1x128 block) and e4m3 activations (power-of-two scale per
                         * row and 32-column block) in the block projections; bf16 in_proj, final layer, attention */

#define T2W_FLAG_GRAPH 1u /* capture the whole solve in a CUDA graph per (layout, buffers) key and replay it */

/* Hyper-parameters (the reference reads them off the estimator module: dit_fast.py:109-114, dit_graph.py:56-60). */
typedef struct t2w_config {
  int32_t mel, hidden, depth, heads, head_dim, ffn, steps, freq_dim;
  float cfg_rate, t_scale, max_period, eps_block, eps_final, eps_qk, eps_conv;
} t2w_config;

/* Weight slots: the `weights` array of t2w_create holds T2W_W_COUNT global pointers followed by depth * T2W_B_COUNT
 * per-block pointers (block b at T2W_W_COUNT + b * T2W_B_COUNT).  Every pointer is fp32 device memory in the
 * reference module's own layout (nn.Linear [out, in], Conv1d [out, in, k]); names are the state-dict paths of
 * stepaudio2's DiT (estimator.<...>). */
enum t2w_weight_slot {
  T2W_W_TEMB_FC1_W = 0, /* t_embedder.mlp.0.weight [H, freq]   */
  T2W_W_TEMB_FC1_B,     /* t_embedder.mlp.0.bias               */
  T2W_W_TEMB_FC2_W,     /* t_embedder.mlp.2.weight [H, H]      */
  T2W_W_TEMB_FC2_B,
  T2W_W_IN_W,           /* in_proj.weight [H, 4 mel]           */
  T2W_W_IN_B,
  T2W_W_FINAL_ADA_W,    /* final_layer.adaLN_modulation.1.weight [2H, H] */
  T2W_W_FINAL_ADA_B,
  T2W_W_FINAL_W,        /* final_layer.linear.weight [mel, H]  */
  T2W_W_FINAL_B,
  T2W_W_COUNT
};
enum t2w_block_slot {
  T2W_B_ADA_W = 0, /* blocks.i.adaLN_modulation.1.weight [9H, H] */
  T2W_B_ADA_B,
  T2W_B_Q_W, T2W_B_Q_B, T2W_B_K_W, T2W_B_K_B, T2W_B_V_W, T2W_B_V_B, /* attn.to_q/to_k/to_v */
  T2W_B_QN_W, T2W_B_QN_B, T2W_B_KN_W, T2W_B_KN_B,                   /* attn.q_norm / k_norm [head_dim] */
  T2W_B_PROJ_W, T2W_B_PROJ_B,                                       /* attn.proj */
  T2W_B_C1_W, T2W_B_C1_B,                                           /* conv.block.1 (Conv1d [H, H, 3]) */
  T2W_B_CLN_W, T2W_B_CLN_B,                                         /* conv.block.3 (LayerNorm [H]) */
  T2W_B_C2_W, T2W_B_C2_B,                                           /* conv.block.6 */
  T2W_B_FC1_W, T2W_B_FC1_B, T2W_B_FC2_W, T2W_B_FC2_B,               /* mlp.fc1 / mlp.fc2 */
  T2W_B_COUNT
};

typedef struct t2w_solver t2w_solver;

/* One packed solve: n_streams requests, stream i = P_i prompt frames then T_i chunk frames (L_i = P_i + T_i).  The
 * token-major inputs concatenate the streams' frames: n_tok = sum L_i rows of `mel` floats.  cond is the prompt mel
 * over prompt frames and zeros over chunk frames; spk is the post-affine speaker vector.  The CFG uncond rows (zero
 * mu / spk / cond) are made on the device.  out receives the final x of every frame (the chunk mel is rows
 * P_i .. L_i - 1 of stream i). */
typedef struct t2w_batch {
  int32_t n_streams;
  const int32_t* prompt_len; /* host [n_streams] */
  const int32_t* chunk_len;  /* host [n_streams] */
  const float* x0;           /* device [n_tok, mel] */
  const float* mu;           /* device [n_tok, mel] */
  const float* cond;         /* device [n_tok, mel] */
  const float* spk;          /* device [n_streams, mel] */
  float* out;                /* device [n_tok, mel] */
} t2w_batch;

/* Library / device probes. */
T2W_API int t2w_version(void);
T2W_API int t2w_device_ok(int device); /* 1 when `device` is an sm_100 GPU the kernels can run on, else 0 */
T2W_API int t2w_last_cuda_error(void); /* the cudaError_t of the last T2W_ERR_CUDA on this thread */

/* Build a solver on the current device: casts / quantises the weights once into solver-owned memory and computes every
 * step's adaLN modulations (t_embedder + adaLN_modulation of each block and the final layer) with the time-embedding
 * kernel.  t_sched: host [2 * steps] fp32 (t, dt) per Euler step as the reference's solver loop produces them
 * (token2wav_batch.py:669-693), or NULL for the cosine schedule evaluated in double.  `stream` orders the set-up work;
 * the call synchronises it before returning.  Every later call that takes the solver (or a slot pool made from it)
 * runs on this device whatever device is current, and leaves the caller's current device as it found it; the
 * pointers and stream passed to those calls must belong to this device. */
T2W_API int t2w_create(const t2w_config* cfg, const float* t_sched, const float* const* weights, int32_t n_weights,
               int32_t precision, void* stream, t2w_solver** out);
T2W_API int t2w_destroy(t2w_solver* s);

/* Workspace bytes a t2w_solve_packed call with these lengths needs (0 on invalid lengths). */
T2W_API size_t t2w_workspace_bytes(const t2w_solver* s, int32_t n_streams, const int32_t* prompt_len, const int32_t* chunk_len);

/* The full S-step CFG Euler solve of a packed batch on `stream` (asynchronous). */
T2W_API int t2w_solve_packed(t2w_solver* s, const t2w_batch* batch, void* workspace, size_t workspace_bytes, uint32_t flags,
                     void* stream);

/* ---- Steady-state (slot-pool) solve: the production form of the same estimator (FastDiT.solve,
 * engine/runtime/dit_fast.py:432-495).  Every cached key frame of a CFG row is one slot of a pool holding K and V of
 * each (step, block); a call solves one window of T_i frames per request against each CFG row's key list (its cached
 * slots followed by the window's new slots, which the call fills), and each CFG row's two cached conv frames per
 * (step, block, conv) sit in a conv-cache row slot.  Slot allocation, the [new, cache] order and the trim to the
 * prompt's frames + 100 stay with the caller (host bookkeeping, as the reference's SlotPool / FastCache). */
typedef struct t2w_slots t2w_slots;

typedef struct t2w_slot_batch {
  int32_t n_streams;       /* requests n */
  const int32_t* chunk_len; /* host [n] window frames T_i > 0 */
  const int32_t* kv_len;    /* host [2n] keys of CFG row r (cond rows 0..n-1, then uncond rows): cached + T_i new */
  const int32_t* kv_idx;    /* host: the 2n key lists (pool slots) concatenated; each ends with its T_i new slots */
  const int32_t* cnn_rd;    /* host [2n] conv-cache row slot each CFG row reads */
  const int32_t* cnn_wr;    /* host [2n] row slot that receives its new conv frames (== rd keeps them) */
  const float* x0;          /* device [sum T, mel] (the flow's fixed noise at each request's cache length) */
  const float* mu;          /* device [sum T, mel] */
  const float* cond;        /* device [sum T, mel] or NULL (zeros) */
  const float* spk;         /* device [n, mel] */
  float* out;               /* device [sum T, mel]: each window's mel, token-major */
} t2w_slot_batch;

/* Pools for n_slots key slots and n_rowslots conv-cache row slots on the solver's device (zeroed):
 * steps * depth * (n_slots * 4 * hidden + n_rowslots * 8 * hidden) bytes. */
T2W_API int t2w_slots_create(const t2w_solver* s, int32_t n_slots, int32_t n_rowslots, t2w_slots** out);
T2W_API int t2w_slots_destroy(t2w_slots* p);
/* K / V of every (step, block): slot src[i] -> dst[i] (host arrays; FastDiT.clone, dit_fast.py:204-216). */
T2W_API int t2w_slots_copy(t2w_slots* p, const int32_t* src, const int32_t* dst, int32_t n, void* stream);
/* Conv caches of every (step, block): row slot src -> dst, or zeros into dst when src < 0 (FastDiT.new_cache). */
T2W_API int t2w_slots_copy_row(t2w_slots* p, int32_t src, int32_t dst, void* stream);
/* The pools' device memory and geometry, for callers that move caches in and out of slots themselves (the module-level
 * forward_chunk(..., cnn_cache, att_cache) adapter, token2wav_batch.py:643-644): kv bf16 [n_sb][n_slots][2 hidden]
 * (slot s of (step, block) sb: K of head h at columns h*64 .. +63, V at hidden + h*64 .. +63), cnn bf16
 * [n_sb][n_rowslots][2 convs][2 frames, oldest first][hidden], n_sb = steps * depth with sb = step * depth + block. */
T2W_API int t2w_slots_pools(const t2w_slots* p, void** kv, void** cnn, int32_t* n_sb, int32_t* n_slots,
                            int32_t* n_rowslots, int32_t* hidden);
/* Workspace bytes of a t2w_solve_slots call (0 on an invalid batch). */
T2W_API size_t t2w_slot_workspace_bytes(const t2w_solver* s, const t2w_slots* p, const t2w_slot_batch* b);
/* The S-step CFG Euler solve of one window per request against the pools (bf16 path).  Attention gathers each CFG
 * row's key list from the pool; the causal convs read the row's cached frames in front of its window.  Asynchronous
 * on `stream`; the host arrays are read before the call returns (they are uploaded into the workspace on `stream`).
 * flags T2W_FLAG_GRAPH: replay a CUDA graph per (sizes of the call's lists, workspace, input / output and pool
 * buffers), captured the second time such a key is seen (the reference's FastDiT.capture, dit_fast.py:347-428);
 * keep the input / output buffers fixed between calls (copy into static buffers) so the key repeats. */
T2W_API int t2w_solve_slots(t2w_solver* s, t2w_slots* p, const t2w_slot_batch* b, void* workspace, size_t workspace_bytes,
                            uint32_t flags, void* stream);

/* ---- Stream caches kept by the library (replaces the reference's Python SlotPool / FastCache bookkeeping,
 * engine/runtime/dit_fast.py:58-97,181-216, and the order / trim after a solve, dit_fast.py:480-490).  A cache is an
 * int32 handle into a registry of the slot pools; per CFG row (0 conditional, 1 unconditional) it holds its key slots
 * in the reference's tensor order (each kept window's keys in front of the older ones) and one conv-cache row slot.
 * After a kept window the order is cut to its first `keep` entries plus its last 100 (token2wav_batch.py:33-39).
 * Slots are handed out by the library; a stale or unknown handle is T2W_ERR_INVALID.  Calls on one t2w_slots are
 * serialised by the library's lock; the GPU work they enqueue is ordered by the caller's stream (slots returned by one
 * call may be written by the next call on the same stream). */
typedef struct t2w_cache_info {
  int32_t length;     /* cached keys per CFG row */
  int32_t keep;       /* trim length */
  int32_t rowslot[2]; /* conv-cache row slot of each CFG row */
} t2w_cache_info;

/* A new empty cache (FastDiT.new_cache, dit_fast.py:181-189): its two conv-cache row slots are zeroed on `stream`.
 * T2W_ERR_EXHAUSTED when no row slots are left. */
T2W_API int t2w_cache_new(t2w_slots* p, int32_t keep, void* stream, int32_t* handle);
/* Return a cache's key and row slots (FastDiT.release, dit_fast.py:189-195); the handle is retired. */
T2W_API int t2w_cache_release(t2w_slots* p, int32_t handle);
/* An independent copy: new slots holding the same keys and values and a copy of the conv caches, enqueued on
 * `stream` (FastDiT.clone, dit_fast.py:204-216). */
T2W_API int t2w_cache_clone(t2w_slots* p, int32_t handle, void* stream, int32_t* out);
T2W_API int t2w_cache_get(const t2w_slots* p, int32_t handle, t2w_cache_info* info);
T2W_API int t2w_cache_set_keep(t2w_slots* p, int32_t handle, int32_t keep);
/* The key slots of CFG row `half` in the reference's order (cap entries at most; returns T2W_ERR_INVALID if fewer). */
T2W_API int t2w_cache_keys(const t2w_slots* p, int32_t handle, int32_t half, int32_t* slots, int32_t cap);
/* Give an EMPTY cache n key slots per CFG row as its order (row 0's ids to slots[0 .. n), row 1's to slots[n .. 2n)),
 * for callers that write keys into those slots themselves (the module-level forward_chunk adapter). */
T2W_API int t2w_cache_reserve(t2w_slots* p, int32_t handle, int32_t n, int32_t* slots);
/* Pool usage: key slots handed out, conv-cache row slots still free, live cache handles. */
T2W_API int t2w_slots_usage(const t2w_slots* p, int32_t* keys_in_use, int32_t* rowslots_free, int32_t* caches);

/* One window per request against the library-kept caches: the steady-state solve with the host bookkeeping done
 * natively.  x0 of request i is temperature * noise[:, L_i : L_i + T_i] (the flow's fixed noise read at the cache
 * length L_i, as FastDiT.solve reads cfm.rand_noise, dit_fast.py:448-449), gathered on the device.  Requests whose
 * keep[i] != 0 keep the window's keys (in front of their order, then trimmed) and conv caches; the others (final
 * flushes) leave their caches as they were. */
typedef struct t2w_cached_batch {
  int32_t n_streams;
  const int32_t* handle;    /* host [n] cache handles, pairwise distinct */
  const int32_t* chunk_len; /* host [n] window frames T_i > 0 */
  const uint8_t* keep;      /* host [n] */
  const float* noise;       /* device [mel, noise_frames] */
  int32_t noise_frames;
  float temperature;
  const float* mu;          /* device [sum T, mel] */
  const float* cond;        /* device [sum T, mel] or NULL (zeros) */
  const float* spk;         /* device [n, mel] */
  float* out;               /* device [sum T, mel] */
} t2w_cached_batch;
T2W_API size_t t2w_cached_workspace_bytes(const t2w_solver* s, const t2w_slots* p, const t2w_cached_batch* b);
/* Asynchronous on `stream`; the caches' records are updated before the call returns.  flags as t2w_solve_slots. */
T2W_API int t2w_solve_cached(t2w_solver* s, t2w_slots* p, const t2w_cached_batch* b, void* workspace,
                             size_t workspace_bytes, uint32_t flags, void* stream);

/* Kernel classes of t2w_profile_solve. */
enum t2w_kernel_class {
  T2W_KC_PACK = 0,   /* input packing (CFG rows) */
  T2W_KC_GEMM_IN,    /* in_proj GEMM */
  T2W_KC_LN_MOD,     /* LayerNorm + adaLN modulation (norm1 / norm3 / norm2 / final) */
  T2W_KC_GEMM_QKV,   /* QKV GEMM with the per-head q / k norms */
  T2W_KC_ATTN,       /* varlen attention */
  T2W_KC_GEMM_PROJ,  /* attention output projection + gated residual */
  T2W_KC_GEMM_CONV1, /* first causal conv (3 taps) */
  T2W_KC_LN_MISH,    /* conv LayerNorm (affine) + Mish */
  T2W_KC_GEMM_CONV2, /* second causal conv + gated residual */
  T2W_KC_GEMM_FC1,   /* MLP fc1 + GELU */
  T2W_KC_GEMM_FC2,   /* MLP fc2 + gated residual */
  T2W_KC_GEMM_FINAL, /* final linear */
  T2W_KC_EULER,      /* CFG combine + Euler step */
  T2W_KC_COUNT
};

/* One eager solve with a CUDA event between consecutive launches; ms[c] / launches[c] receive each kernel class's
 * summed device time and launch count ([T2W_KC_COUNT] each).  Synchronises `stream`. */
T2W_API int t2w_profile_solve(t2w_solver* s, const t2w_batch* batch, void* workspace, size_t workspace_bytes, void* stream,
                              float* ms, int32_t* launches);

/* Synchronise the solver's error word: T2W_OK, or T2W_ERR_TIMEOUT if a kernel gave up on a wait (then cleared). */
T2W_API int t2w_check(t2w_solver* s);

/* Test entry point of the bounded waits (no reference counterpart; the reference's analogue is failure isolation,
 * engine/runtime/t2w_worker.py:546-553): launches the row kernel in its early-start mode on 256 scratch rows whose
 * 128-row block counter nothing publishes, with the wait limited to limit_ns (1e5 .. 2e9).  Every warp gives up after
 * the limit and records T2W_ERR_TIMEOUT in the solver's error word, then returns; t2w_check reports and clears it.
 * Asynchronous on `stream`; the solver stays usable. */
T2W_API int t2w_test_wait_timeout(t2w_solver* s, int64_t limit_ns, void* stream);

/* Copy the solver's modulation tables to device memory: mods [steps, depth, 9, H] (order sh_msa, 1+sc_msa, g_msa,
 * sh_mlp, 1+sc_mlp, g_mlp, sh_conv, 1+sc_conv, g_conv) and final [steps, 2, H] (sh, 1+sc); dts [steps] fp32. */
T2W_API int t2w_mods(const t2w_solver* s, float* mods, float* final_mods, float* dts, void* stream);

/* Counters: graph replays, graph captures, eager solves. */
T2W_API int t2w_counts(const t2w_solver* s, int64_t* graph_replays, int64_t* graph_captures, int64_t* eager_solves);

/* ---- single kernels (test entry points; bf16 buffers are passed as void*) ---------------------------------------- */

/* out[r] = bf16(LN(h[r]) * scale1 + shift) (LayerNorm without affine, fp32 math); rows whose pad[r] != 0 are zero. */
T2W_API int t2w_ln_mod(const float* h, int32_t ld_h, const float* shift, const float* scale1, float eps, int32_t rows,
               int32_t C, void* out_bf16, int32_t ld_out, const uint8_t* pad, void* stream);

/* h[r] += g * y[r] (y bf16 [rows, C], fp32 math, h updated in place; skipped when y is NULL), then
 * out[r] = bf16(LN(h[r]) * scale1 + shift); rows whose pad[r] != 0 get zero output.  Replaces add_ln_mod
 * (dit_kernels.py:35-60), with the residual kept in fp32. */
T2W_API int t2w_add_ln_mod(float* h, const void* y_bf16, const float* g, const float* shift, const float* scale1, float eps,
                           int32_t rows, int32_t C, void* out_bf16, const uint8_t* pad, void* stream);

/* out[r] = bf16(Mish(LN_affine(x[r]))) with x bf16; rows whose pad[r] != 0 are zero. */
T2W_API int t2w_ln_mish(const void* x_bf16, const float* w, const float* b, float eps, int32_t rows, int32_t C,
                void* out_bf16, const uint8_t* pad, void* stream);

#define T2W_EPI_F32 0  /* out fp32 = acc + bias */
#define T2W_EPI_BF16 1 /* out bf16 = acc + bias */
#define T2W_EPI_GELU 2 /* out bf16 = gelu_tanh(acc + bias) */
#define T2W_EPI_RESID 3 /* out fp32 += gate * (acc + bias), in place: the gated residual (gate: N floats, qk[0]) */
#define T2W_EPI_QKV 4  /* out bf16 = [LN_q(q) | LN_k(k) | v] per 64-wide head (q/k affine norms) */
#define T2W_EPI_SILU 5 /* out bf16 = silu(acc + bias): the flow encoder's swish feed-forward */
#define T2W_EPI_LEAKY 6 /* out bf16 = leaky_relu(acc + bias) with slope qk_eps: the pre-lookahead conv1 */
#define T2W_EPI_GELU_FP8 8 /* t2w_gemm_e4m3 only: out e4m3 = gelu_tanh(acc + bias) with its scale atoms */

/* C[M, N] = sum_tap A[m + tap_row0 + tap, :K] . W[n, tap*K : (tap+1)*K] then the epilogue.  A bf16 [rows_a, lda],
 * W bf16 [N, taps*K]; rows outside [0, rows_a) read as zero (causal-conv taps).  M % 128 == 0, K % 64 == 0,
 * N % 128 == 0 or N == 80.  qk: for T2W_EPI_QKV, [qn_w, qn_b, kn_w, kn_b] (head_dim each) and qk_eps; q columns
 * [0, N/3), k [N/3, 2N/3).  qk: for T2W_EPI_RESID, qk[0] is the gate (N floats); out, gate and bias 16-byte aligned.
 * The solve applies the gated residual of proj with T2W_EPI_RESID; those of conv2 / fc2 are added from their bf16
 * outputs by t2w_add_ln_mod. */
T2W_API int t2w_gemm(const void* A_bf16, int32_t lda, int32_t rows_a, const void* W_bf16, const float* bias, int32_t M,
                     int32_t N, int32_t K, int32_t taps, int32_t tap_row0, int32_t epi, void* out, int32_t ldo,
                     const float* const* qk, float qk_eps, void* stream);

/* Varlen attention over packed sequences with the block-causal chunk mask: sequence s has its keys at rows
 * seq_row[s] .. seq_row[s] + seq_len[s] - 1 of qkv (bf16 [rows, 3 * heads * 64], q | k | v column blocks); a query at
 * position i attends keys j < (i < prompt_len[s] ? prompt_len[s] : seq_len[s]).  out bf16 [rows, heads * 64].
 * seq_row / seq_len / prompt_len are host arrays.  The per-call work list is uploaded from host memory that lives only
 * for the call, so a stream under capture is refused (T2W_ERR_INVALID, nothing enqueued). */
T2W_API int t2w_attn_varlen(const void* qkv_bf16, int32_t rows, int32_t heads, int32_t n_seq, const int32_t* seq_row,
                    const int32_t* seq_len, const int32_t* prompt_len, void* out_bf16, void* stream);

/* t2w_attn_varlen for callers that cannot allocate device memory when they call in (a runtime that has reserved the
 * whole GPU for its own pool, or a plugin running where the CUDA allocator must not be called).  No counterpart in the
 * reference.  Same arguments, same results; the per-call work list (one entry per 128-query tile) lives in a fixed
 * device array of this library instead of a per-call allocation: at most 8192 tiles per call (160 KB, held on every GPU
 * that loads the library until exit); more returns T2W_ERR_INVALID.  The first call on a device looks up that array's
 * device address.  Like t2w_attn_varlen, it uploads the work list from host memory that lives only for the call, so no
 * call may be made on a stream under capture: such a call returns T2W_ERR_INVALID and enqueues nothing.  All calls
 * share the array: calls whose GPU work overlaps (two streams, two threads) race on it and must be serialised by the
 * caller. */
T2W_API int t2w_attn_varlen_noalloc(const void* qkv_bf16, int32_t rows, int32_t heads, int32_t n_seq,
                                    const int32_t* seq_row, const int32_t* seq_len, const int32_t* prompt_len,
                                    void* out_bf16, void* stream);

/* ---- FP8 (e4m3) path: values in e4m3 with one power-of-two (UE8M0) scale per row and 32-column block.
 * The scales of a [rows, C] matrix are stored as "atoms": one 512-byte atom per (128-row tile, 128-column block),
 * atom (r / 128) * (C / 128) + j / 4 holding row r's scale of block j at byte (r % 32) * 16 + (r % 128 / 32) * 4 + j % 4
 * (the layout the tensor core's scale-factor copy reads).  A "row-shifted layout" d stores row r at position r + d;
 * the causal conv's GEMM reads layouts d = 0, 1, 2, which the producing kernel writes together (n_layouts = 3,
 * layout d at sf + d * layout_bytes).  The reference quantises its FP8 linears with per-output-row weight scales and
 * per-token activation scales (engine/runtime/fp8.py:15-40); these entry points use per-block power-of-two scales,
 * which the block-scaled MMA applies inside the K loop. */

/* Bytes of one layout of scale atoms for a [rows, C] e4m3 matrix (C % 128 == 0). */
T2W_API size_t t2w_e4m3_sf_bytes(int32_t rows, int32_t C);
/* bf16 [rows, C] -> e4m3 [rows, C] + scale atoms (per 1 x 32 block; C = 128, 512, 1536 or 2048). */
T2W_API int t2w_quant_e4m3(const void* x_bf16, int32_t rows, int32_t C, void* out_e4m3, uint8_t* sf, int32_t n_layouts,
                           int64_t layout_bytes, void* stream);
/* fp32 weight [N, Kt] -> e4m3 [N, Kt] + one power-of-two scale per 1 x 128 block, as atoms [Kt / 128][N / 128][512]
 * (the weight layout t2w_gemm_e4m3 reads; N, Kt multiples of 128). */
T2W_API int t2w_quant_weight_e4m3(const float* w, int32_t N, int32_t Kt, void* w_e4m3, uint8_t* sf, void* stream);
/* t2w_add_ln_mod / t2w_ln_mish with e4m3 output and its scale atoms (n_layouts 1-3). */
T2W_API int t2w_add_ln_mod_e4m3(float* h, const void* y_bf16, const float* g, const float* shift, const float* scale1,
                                float eps, int32_t rows, int32_t C, void* out_e4m3, uint8_t* sf, int32_t n_layouts,
                                int64_t layout_bytes, const uint8_t* pad, void* stream);
T2W_API int t2w_ln_mish_e4m3(const void* x_bf16, const float* w, const float* b, float eps, int32_t rows, int32_t C,
                             void* out_e4m3, uint8_t* sf, int32_t n_layouts, int64_t layout_bytes, const uint8_t* pad,
                             void* stream);
/* t2w_attn_varlen with e4m3 output [rows, heads * 64] and its scale atoms (layout 0). */
T2W_API int t2w_attn_varlen_e4m3(const void* qkv_bf16, int32_t rows, int32_t heads, int32_t n_seq, const int32_t* seq_row,
                                 const int32_t* seq_len, const int32_t* prompt_len, void* out_e4m3, uint8_t* sf,
                                 void* stream);
/* Block-scaled FP8 GEMM: C[M, N] = sum_tap dequant(A8)[m + tap_row0 + tap, :K] . dequant(W8)[n, tap*K : (tap+1)*K]^T
 * then the epilogue (T2W_EPI_BF16, T2W_EPI_QKV: bf16 out [M, ldo]; T2W_EPI_GELU_FP8: e4m3 out + out_sf atoms).
 * A8 e4m3 [rows_a, lda bytes] with scale atoms sfa in sfa_layouts row-shifted layouts (tap t reads layout
 * -(tap_row0 + t)); W8 and sfw from t2w_quant_weight_e4m3.  M % 128 == 0, N % 256 == 0, K % 128 == 0; fp32
 * accumulation in TMEM.  Replaces the reference's fp8_linear (engine/runtime/fp8.py:27-36). */
T2W_API int t2w_gemm_e4m3(const void* A8, int32_t lda, int32_t rows_a, const uint8_t* sfa, int32_t sfa_layouts,
                          int64_t sfa_layout_bytes, const void* W8, const uint8_t* sfw, const float* bias, int32_t M,
                          int32_t N, int32_t K, int32_t taps, int32_t tap_row0, int32_t epi, void* out, int32_t ldo,
                          uint8_t* out_sf, const float* const* qk, float qk_eps, void* stream);

/* x[i] += dt ((1 + w) dphi[row[i]] - w dphi[row[i] + half_rows]) for the n_tok cond tokens (mel floats each); also
 * writes bf16(x) into hx[row] and hx[row + half_rows] (first mel columns of ld_hx) and, when out != NULL, out[i] = x. */
T2W_API int t2w_euler_cfg(float* x, const float* dphi, int32_t ld_dphi, const int32_t* tok_row, int32_t n_tok, int32_t mel,
                  int32_t half_rows, float dt, float w, void* hx_bf16, int32_t ld_hx, float* out, void* stream);

/* ---- Flow encoder: the step before the solve (speech tokens -> mu).
 *
 * Replaces the flow encoder's chunk forward as the engine drives it (paths inside the reference):
 *   t2w_encoder_create    the flow module's input_embedding, encoder (UpsampleConformerEncoderV2) and encoder_proj,
 *                         weights cast once (the engine runs them in its activation dtype, token2wav_batch.py:184-206)
 *   t2w_encode            BatchedToken2Wav._flow_encode + _encoder + _encoder_core + encoder_proj, and the cache trim
 *                         of _flow_finish (token2wav_batch.py:42-79,365-399,402-478); a prompt setup
 *                         (_setup_encoder_one / _setup_encoder_batched, token2wav_batch.py:556-616) is a window of a
 *                         new stream with empty caches (its tokens plus the look-ahead silence tokens)
 *   t2w_enc_stream_*      the per-stream flow_cache entries conformer_cnn_cache / conformer_att_cache
 *                         (token2wav_batch.py:408-444): kept natively as key-slot lists over per-layer K/V pools
 * Every window of a call has its own token count, cache length and final flag, so final windows never need the
 * reference's merged-call padding (token2wav_batch.py:365-386). */
typedef struct t2w_enc_config {
  int32_t vocab, hidden, heads, head_dim, ffn, blocks1, blocks2, stride, lookahead, mel;
  float eps_layer, eps_embed, eps_after, leaky_slope, max_period;
} t2w_enc_config;

/* Weight slots of t2w_encoder_create: T2W_E_COUNT global pointers, then (blocks1 + blocks2) * T2W_EL_COUNT per-layer
 * pointers (encoders.0 .. encoders.{blocks1-1}, then up_encoders.0 ..; layer l at T2W_E_COUNT + l * T2W_EL_COUNT).
 * fp32 device memory in the module's layout; names are the flow module's state-dict paths. */
enum t2w_enc_weight_slot {
  T2W_E_EMB = 0,                    /* input_embedding.weight [vocab, hidden] */
  T2W_E_EMBED_W, T2W_E_EMBED_B,     /* encoder.embed.out.0 (Linear hidden -> hidden) */
  T2W_E_EMBED_LN_W, T2W_E_EMBED_LN_B, /* encoder.embed.out.1 (LayerNorm, eps_embed) */
  T2W_E_PL_C1_W, T2W_E_PL_C1_B,     /* encoder.pre_lookahead_layer.conv1 [hidden, hidden, lookahead + 1] */
  T2W_E_PL_C2_W, T2W_E_PL_C2_B,     /* encoder.pre_lookahead_layer.conv2 [hidden, hidden, 3] */
  T2W_E_UP_W, T2W_E_UP_B,           /* encoder.up_layer.conv [hidden, hidden, 2 stride + 1] */
  T2W_E_UPEMB_W, T2W_E_UPEMB_B,     /* encoder.up_embed.out.0 */
  T2W_E_UPEMB_LN_W, T2W_E_UPEMB_LN_B, /* encoder.up_embed.out.1 */
  T2W_E_AFTER_W, T2W_E_AFTER_B,     /* encoder.after_norm (eps_after) */
  T2W_E_PROJ_W, T2W_E_PROJ_B,       /* encoder_proj [mel, hidden] */
  T2W_E_COUNT
};
enum t2w_enc_layer_slot {
  T2W_EL_Q_W = 0, T2W_EL_Q_B, T2W_EL_K_W, T2W_EL_K_B, T2W_EL_V_W, T2W_EL_V_B, /* self_attn.linear_q / _k / _v */
  T2W_EL_OUT_W, T2W_EL_OUT_B,       /* self_attn.linear_out */
  T2W_EL_POS_W,                     /* self_attn.linear_pos.weight [hidden, hidden] (no bias) */
  T2W_EL_POS_U, T2W_EL_POS_V,       /* self_attn.pos_bias_u / pos_bias_v [heads, head_dim] */
  T2W_EL_FF1_W, T2W_EL_FF1_B, T2W_EL_FF2_W, T2W_EL_FF2_B, /* feed_forward.w_1 / w_2 */
  T2W_EL_NMHA_W, T2W_EL_NMHA_B, T2W_EL_NFF_W, T2W_EL_NFF_B, /* norm_mha / norm_ff (eps_layer) */
  T2W_EL_COUNT
};

typedef struct t2w_encoder t2w_encoder;

/* Build an encoder on the current device.  max_frames bounds a window's frames and every attention's key count after
 * the upsampling (a stream's second-stack cache plus stride * its window), and sizes the relative-position tables
 * (linear_pos of the sinusoid at every relative position -(max_frames - 1) .. max_frames - 1, computed once here in
 * fp32 and stored bf16).  n_slots1 / n_slots2: key slots of each first- / second-stack layer's K/V pool; n_streams:
 * live streams at most.  `stream` orders the set-up work; the call synchronises it before returning. */
T2W_API int t2w_encoder_create(const t2w_enc_config* cfg, const float* const* weights, int32_t n_weights,
                               int32_t max_frames, int32_t n_slots1, int32_t n_slots2, int32_t n_streams, void* stream,
                               t2w_encoder** out);
T2W_API int t2w_encoder_destroy(t2w_encoder* e);

/* A stream with empty caches (a prompt setup's state: no keys, zero conv caches, zeroed on `stream`) and trim length
 * `keep` (the prompt's mel frames, stride * its tokens).  T2W_ERR_EXHAUSTED when n_streams are live. */
T2W_API int t2w_enc_stream_new(t2w_encoder* e, int32_t keep, void* stream, int32_t* handle);
T2W_API int t2w_enc_stream_release(t2w_encoder* e, int32_t handle);
/* A new stream holding a copy of a stream's caches (keys in new slots of every layer's pool, the conv-cache frames,
 * keep), enqueued on `stream`: the copy a request's stream takes of its prompt's flow_cache when the prompt is not
 * adopted (BatchedToken2Wav.new_stream, token2wav_batch.py:267-279). */
T2W_API int t2w_enc_stream_clone(t2w_encoder* e, int32_t handle, void* stream, int32_t* out);
/* Cached key frames of the first and second stack (the reference cache's time length is 2 * keys1 = keys2 after a
 * setup; see t2w_encode for how they advance) and the trim length. */
T2W_API int t2w_enc_stream_get(const t2w_encoder* e, int32_t handle, int32_t* keys1, int32_t* keys2, int32_t* keep);
/* Key slots in use in the first- and second-stack pools, live streams. */
T2W_API int t2w_enc_usage(const t2w_encoder* e, int32_t* slots1, int32_t* slots2, int32_t* streams);

/* One window per stream.  Window i has n_tokens[i] tokens: its T_i = n_tokens[i] - lookahead frames plus the
 * look-ahead tokens, or, when final[i] != 0, T_i = n_tokens[i] frames followed by `lookahead` zero frames (the
 * reference's last_chunk padding).  A window whose caches are kept (final[i] == 0) needs T_i >= 2.  mu receives
 * stride * T_i rows of `mel` floats per window, windows in call order (encoder_proj of the after_norm output,
 * token-major: the rows t2w_solve_cached takes as mu).  After the call each stream's caches have advanced as the
 * reference advances them: conv caches = the last frames of [cache | new]; first stack keys = the first
 * min(K1, (keep + 100) / 2) of [cached | new] when 2 K1 > keep + 100, else all K1 (the reference's first-stack
 * cache is tiled twice along time, cut to its first keep and last 100 frames, and read back as the first half);
 * second stack keys = [cached | new] cut to the first keep and last 100 (token2wav_batch.py:33-39,395).
 * tokens: host, the windows' tokens concatenated (each < vocab).  Asynchronous on `stream`; the host arrays are read
 * before the call returns. */
typedef struct t2w_enc_batch {
  int32_t n_streams;
  const int32_t* handle;   /* host [n] stream handles, pairwise distinct */
  const int32_t* n_tokens; /* host [n] */
  const uint8_t* final;    /* host [n] */
  const int32_t* tokens;   /* host [sum n_tokens] */
  float* mu;               /* device [sum stride * T_i, mel] */
} t2w_enc_batch;
T2W_API size_t t2w_enc_workspace_bytes(const t2w_encoder* e, const t2w_enc_batch* b);
/* flags T2W_FLAG_GRAPH: replay a CUDA graph per launch structure (the sizes of the call's lists, the workspace and mu
 * buffers), captured the second time such a key is seen (the reference captures its encoder per bucket,
 * EncoderGraphs, token2wav_batch.py:206,413); keep the workspace and mu buffers fixed between calls so keys repeat.
 * A stream under capture with T2W_FLAG_GRAPH is refused (T2W_ERR_INVALID). */
T2W_API int t2w_encode(t2w_encoder* e, const t2w_enc_batch* b, void* workspace, size_t workspace_bytes, uint32_t flags,
                       void* stream);
/* Counters: graph replays, graph captures, eager calls. */
T2W_API int t2w_enc_counts(const t2w_encoder* e, int64_t* replays, int64_t* captures, int64_t* eager);
/* Synchronise the encoder's error word: T2W_OK, or T2W_ERR_TIMEOUT if a kernel gave up on a wait (then cleared). */
T2W_API int t2w_enc_check(t2w_encoder* e);

/* Single encoder kernels (test entry points).
 * Relative-position attention (RelPositionMultiHeadedAttention of the conformer layers with the zero-pad rel_shift):
 * for sequence s with T queries at rows q_row[s] .. of qkv4 (bf16 [rows, 4 H]: [q + pos_bias_u | q + pos_bias_v | k | v]
 * per row, H = heads * 64) and K keys, key j from pool row kv_idx[kv_off[s] + j] (bf16 [pool_rows, 2 H]: [k | v]),
 * query i at position K - T + i: score = ((q_i + u) . k_j + (q_i + v) . P[(K - T + i) - j]) / 8 over all K keys, with
 * P the relative-position table (bf16 [2 max_frames - 1, H], row r + max_frames - 1 = linear_pos(pe(r))).
 * out bf16 [rows, H].  q_row / T / K / kv_off: host [n_seq]; kv_idx: host [n_idx].  They are copied from host memory
 * that lives only for the call, so a stream under capture is refused (T2W_ERR_INVALID, nothing enqueued). */
T2W_API int t2w_enc_relattn(const void* qkv4_bf16, int32_t rows, int32_t heads, const void* pool_bf16, int32_t pool_rows,
                            const void* pos_bf16, int32_t max_frames, int32_t n_seq, const int32_t* q_row,
                            const int32_t* T, const int32_t* K, const int32_t* kv_off, const int32_t* kv_idx,
                            int32_t n_idx, void* out_bf16, void* stream);
/* The relative-position table of t2w_encoder_create: pos[r + max_frames - 1] = bf16(W pe(r)) for |r| < max_frames,
 * W fp32 [H, H] (linear_pos.weight), pe(r) = [sin(r w_0), cos(r w_0), sin(r w_1), ...], w_m = max_period^(-2m / H). */
T2W_API int t2w_enc_pos_table(const float* w, int32_t H, int32_t max_frames, float max_period, void* pos_bf16,
                              void* stream);
/* Row LayerNorm of the encoder: y = LN(x) * w + b (eps; w, b fp32 [C]) for fp32 x [rows, C]; writes fp32 y into
 * out_f32 (may alias x) and / or bf16 y into out_bf16 (either may be NULL); rows whose pad[r] != 0 get zeros. */
T2W_API int t2w_enc_ln(const float* x, const float* w, const float* b, float eps, int32_t rows, int32_t C, float* out_f32,
                       void* out_bf16, const uint8_t* pad, void* stream);

/* ---- HiFT vocoder: the step after the solve (mel -> 24 kHz waveform).
 *
 * Replaces (paths inside the reference):
 *   t2w_hift_create      the flow's HiFTGenerator as Token2Wav loads it (engine/models/token2wav.py:249-264; weight
 *                        normalisation folded into plain weights, as the reference's lean form does once)
 *   t2w_vocode           BatchedToken2Wav._vocode (engine/runtime/token2wav_batch.py:813-848) over hift_forward /
 *                        hift_forward_noise / _hift_decode / istft_overlap_add (engine/models/token2wav.py:112-245):
 *                        each window's mel after its stream's 8 cached frames, f0 predictor, harmonic source, the
 *                        decoder, the inverse STFT, the Hamming cross-fade with the previous window, the caches, and
 *                        the output samples (the last 3840 held back unless the window is final; a stream's first
 *                        window starts with 3840 samples of silence)
 *   t2w_hift_stream_*    a stream's hift_cache (mel / source / speech tails, token2wav.py:287-292), kept in the library
 * Strict fp32 (the reference runs Token2Wav with TF32 off: token2wav.py:44-57) unless tf32 is set. */
typedef struct t2w_hift_config {
  int32_t mel, channels, f0_channels, f0_layers, harmonics, sample_rate, n_fft, hop;
  int32_t up_rates[3], up_kernels[3], res_kernels[3], source_kernels[3], dilations[3];
  float nsf_alpha, nsf_sigma, voiced_threshold, lrelu_slope, audio_limit;
  int32_t tf32; /* 0: strict fp32 everywhere (CUDA cores); 2: every convolution on the tensor cores in split form
                 * (3xTF32: operands as pairs of TF32 values, hi W_hi + hi W_lo + lo W_hi; fp32-level products, the
                 * reference's strict-fp32 numerics at tensor-core speed; tf32_parts ignored);
                 * 1: the upsampling stages (transposed convs, source and main ResBlocks) on
                 * TF32 tensor cores, the reference's decode_tf32 option (token2wav.py:160-210); the f0 predictor,
                 * conv_pre and conv_post stay at fp32 level (on the tensor cores: the split form, or the mel rows
                 * tripled as [hi | lo | hi] against [W_hi | W_hi | W_lo]), the source on CUDA cores */
  uint32_t tf32_parts; /* with tf32 set: which parts run on TF32, bit 3 s + p for stage s (0-2) and part p (0 the
                        * transposed conv, 1 the source branch, 2 the ResBlocks) — the reference's per-stage lists
                        * (tf32_stages, token2wav.py:145-158); 0 means every part (tf32 = 1 alone); the parts left out
                        * run in fp32 on CUDA cores */
} t2w_hift_config;

typedef struct t2w_hift t2w_hift;

/* Weight order of t2w_hift_create (fp32 device pointers in the module's layouts; Conv1d [out, in, k],
 * ConvTranspose1d [in, out, k]; state-dict paths of HiFTGenerator):
 *   f0_predictor.condnet.{2l}.weight / .bias for l < f0_layers; f0_predictor.classifier.weight / .bias;
 *   m_source.l_linear.weight / .bias; conv_pre.weight / .bias; ups.{0,1,2}.weight / .bias;
 *   per stage s = 0..2: source_downs.s.weight / .bias, then source_resblocks.s: convs1.{0,1,2}.weight / .bias,
 *     convs2.{0,1,2}.weight / .bias, activations1.{0,1,2}.alpha, activations2.{0,1,2}.alpha;
 *   resblocks.{0..8} (stage s, kernel j at 3 s + j) in the same per-block order; conv_post.weight / .bias.
 * max_frames bounds a window's mel frames (with the 8 cached ones, at most 512); n_streams: live streams at most. */
T2W_API int t2w_hift_create(const t2w_hift_config* cfg, const float* const* weights, int32_t n_weights,
                            int32_t max_frames, int32_t n_streams, t2w_hift** out);
T2W_API int t2w_hift_destroy(t2w_hift* h);
/* Synchronise the vocoder's error word: T2W_OK, or T2W_ERR_TIMEOUT if a kernel gave up on a wait (then cleared). */
T2W_API int t2w_hift_check(t2w_hift* h);
/* A stream with empty caches (its first window has no cached mel frames, source or speech). */
T2W_API int t2w_hift_stream_new(t2w_hift* h, int32_t* handle);
T2W_API int t2w_hift_stream_release(t2w_hift* h, int32_t handle);

typedef struct t2w_vocode_batch {
  int32_t n_streams;
  const int32_t* handle;   /* host [n] stream handles, pairwise distinct */
  const int32_t* T;        /* host [n] window mel frames (a window that is not final needs T >= 8 on its first call) */
  const uint8_t* last;     /* host [n] final window */
  const float* mel;        /* device [sum T, mel] fp32, token-major (the solve's output rows) */
  const float* rand_ini;   /* device [n, harmonics + 1]: the source's initial phases (no effect on the output: the
                            * reference's linear downsampling of the phase increments never reads sample 0) */
  const float* noise;      /* device: per window [harmonics + 1][480 F_i] (channel-major, the reference's draw), windows
                            * concatenated; F_i = T_i plus the 8 cached frames after a stream's first window */
  float* out;              /* device [t2w_vocode_samples]: each window's output samples, windows in order */
  float* source;           /* device [sum 480 F_i] or NULL: the windows' source signals */
  float* speech;           /* device [sum 480 F_i] or NULL: the windows' full speech (after the cross-fade) */
  uint32_t flags;          /* T2W_FLAG_GRAPH: replay a CUDA graph per launch structure (the call's sizes: stream count,
                            * frames, samples), captured the second time a structure is seen; the mel and noise are
                            * copied into the graph's own workspace first and the samples out of it after (the
                            * reference's t2w_graphs option, HiFTGraphs, engine/runtime/hift_graph.py:22-88).  Calls
                            * replaying one graph must be ordered on the GPU (one stream, or synchronised); a caller
                            * that is itself capturing passes 0. */
  void* noise_ready;       /* a cudaEvent_t, or NULL: the call waits for it (on `stream`) before it first reads `noise`,
                            * so the caller may draw the noise on another stream while the call's first kernels (mel
                            * input, conv_pre, the f0 predictor) run. */
} t2w_vocode_batch;
/* Output samples of a call (the sum), per window (per_stream, may be NULL) and each window's frames F_i (frames, may
 * be NULL); -1 on an invalid batch. */
T2W_API int64_t t2w_vocode_samples(const t2w_hift* h, int32_t n, const int32_t* handle, const int32_t* T,
                                   const uint8_t* last, int64_t* per_stream, int32_t* frames);
/* One window per stream; asynchronous on `stream` (the call's scratch is a stream-ordered allocation). */
T2W_API int t2w_vocode(t2w_hift* h, const t2w_vocode_batch* b, void* stream);
/* Counters: graph replays, graph captures, eager calls. */
T2W_API int t2w_hift_counts(const t2w_hift* h, int64_t* graph_replays, int64_t* graph_captures, int64_t* eager_calls);

/* Test entry: one launch of the vocoder's tensor-core convolution (the kernel behind the tf32 stages and the split-form
 * layers), for numerics tests against a plain fp32 / fp64 convolution.
 *   out[row_mul m + row_add, n] = epi(bias[n] + sum_tap sum_c A[m + tap_row0 + tap dil, c] W[n, tap Cin + c]),
 * m < M (M % 128 == 0), A rows outside [0, rows_a) read as zero, rows with pad[row_mul m + row_add] != 0 written as zero
 * (epi 0 bias, 1 Snake with alpha / inv, 3 ELU) or left as they are (2: out += ...); with epi 0 or 2 and out2 != NULL
 * Snake(out) into out2 too.  Cin % 4 == 0, W [N, taps Cp] with Cp = Cin rounded up to 32 (the columns past Cin zero);
 * N % 128 == 0, 64 or 32.  split_in (Cin % 32 == 0): A rows are [hi | lo] (2 Cin floats) and W has [W_hi | W_lo | W_hi]
 * per tap (3 Cin columns); split_out: the output rows are written as [hi | lo] (2 N floats).
 * Asynchronous on `stream`; a bounded wait that gives up writes T2W_ERR_TIMEOUT into *err (device int). */
typedef struct t2w_tconv_args {
  const float* A;
  int32_t lda, rows_a;
  const float* W;
  const float* bias;
  int32_t M, N, Cin, taps, tap_row0, dil;
  float* out;
  int64_t ldo;
  int32_t row_mul, row_add;
  const uint8_t* pad;
  int32_t epi;
  const float* alpha;
  const float* inv;
  float* out2;
  int32_t split_in, split_out;
  int32_t* err;
  const float* resid_in; /* epi 2: out = resid_in + ... (padding rows copied from resid_in); NULL: out in place */
} t2w_tconv_args;
T2W_API int t2w_test_tconv(const t2w_tconv_args* a, void* stream);

/* Test entry: one launch of the slot-pool (gathered-key) attention the steady-state solve runs, for numerics tests.
 * work: host [n_work][5] (q_row, k_row, q_pos, P, L): the queries q_row .. q_row + P - q_pos - 1 of qkv (bf16 [rows,
 * 3 heads 64]) attend the L keys pool[kv_idx[k_row + j]] (K at column h 64, V at heads 64 + h 64 of bf16 rows of
 * pool_ld); out bf16 [rows, heads 64].  kv_idx: host [n_idx], every entry < pool_rows.  pair != 0: the paired form
 * (two items per 128-row tile; every item's queries within 64 rows).  Synchronises the stream. */
T2W_API int t2w_test_attn_gathered(const void* qkv_bf16, int32_t rows, int32_t heads, int32_t n_work, const int32_t* work,
                                   const void* pool_bf16, int32_t pool_rows, int32_t pool_ld, const int32_t* kv_idx,
                                   int32_t n_idx, int32_t pair, void* out_bf16, int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* T2W_B200_H_ */
