// torch custom ops over the C ABI of libt2w_b200.so: torch.ops.b200t2w.*.
//
// The reference engine calls its solver from torch code (BatchedToken2Wav -> FastDiT.solve,
// engine/runtime/token2wav_batch.py:335,356-357,518-519,549 -> engine/runtime/dit_fast.py:432-495).  These ops give
// that call site the B200 solve as registered torch operators (and the flow encoder before it, _flow_encode / _encoder,
// token2wav_batch.py:365-478): tensors in, the current torch CUDA stream of the
// tensors' device as the stream, a C-ABI call, and a RuntimeError carrying the status on failure.  No logic lives here:
// every op is argument conversion around one t2w_* call (include/t2w_b200.h).  Solver and slot-pool objects cross the
// boundary as int handles (their addresses), as the ctypes binding passes them.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <string>
#include <vector>

#include "t2w_b200.h"

namespace {

void check(const char* fn, int rc) {
  TORCH_CHECK(rc == T2W_OK, fn, " failed: status ", rc,
              rc == T2W_ERR_CUDA ? " (cudaError " + std::to_string(t2w_last_cuda_error()) + ")" : std::string());
}

void* stream_of(const at::Tensor& t) {
  TORCH_CHECK(t.is_cuda(), "b200t2w ops take CUDA tensors");
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

std::vector<int32_t> i32(c10::IntArrayRef v) { return std::vector<int32_t>(v.begin(), v.end()); }

template <class T>
T* handle(int64_t h) {
  return reinterpret_cast<T*>(static_cast<intptr_t>(h));
}

const void* ptr(const std::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// ---- solver objects ------------------------------------------------------------------------------------------------

int64_t create(c10::IntArrayRef cfg_i, c10::ArrayRef<double> cfg_f, c10::ArrayRef<double> t_sched, at::TensorList weights,
               int64_t precision) {
  TORCH_CHECK(cfg_i.size() == 8 && cfg_f.size() == 7, "create: 8 integer and 7 float config fields");
  TORCH_CHECK(!weights.empty(), "create: no weights");
  t2w_config c{};
  c.mel = (int32_t)cfg_i[0];
  c.hidden = (int32_t)cfg_i[1];
  c.depth = (int32_t)cfg_i[2];
  c.heads = (int32_t)cfg_i[3];
  c.head_dim = (int32_t)cfg_i[4];
  c.ffn = (int32_t)cfg_i[5];
  c.steps = (int32_t)cfg_i[6];
  c.freq_dim = (int32_t)cfg_i[7];
  c.cfg_rate = (float)cfg_f[0];
  c.t_scale = (float)cfg_f[1];
  c.max_period = (float)cfg_f[2];
  c.eps_block = (float)cfg_f[3];
  c.eps_final = (float)cfg_f[4];
  c.eps_qk = (float)cfg_f[5];
  c.eps_conv = (float)cfg_f[6];
  std::vector<float> ts(t_sched.begin(), t_sched.end());
  std::vector<const float*> w;
  for (const at::Tensor& t : weights) {
    TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous(), "create: weights are contiguous fp32");
    w.push_back(t.data_ptr<float>());
  }
  t2w_solver* s = nullptr;
  check("t2w_create", t2w_create(&c, ts.empty() ? nullptr : ts.data(), w.data(), (int32_t)w.size(), (int32_t)precision,
                                 stream_of(weights[0]), &s));
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(s));
}

void destroy(int64_t solver) { check("t2w_destroy", t2w_destroy(handle<t2w_solver>(solver))); }

int64_t workspace_bytes(int64_t solver, c10::IntArrayRef prompt_len, c10::IntArrayRef chunk_len) {
  TORCH_CHECK(prompt_len.size() == chunk_len.size(), "workspace_bytes: one prompt and chunk length per stream");
  const std::vector<int32_t> P = i32(prompt_len), T = i32(chunk_len);
  return (int64_t)t2w_workspace_bytes(handle<t2w_solver>(solver), (int32_t)P.size(), P.data(), T.data());
}

void solve_packed(int64_t solver, c10::IntArrayRef prompt_len, c10::IntArrayRef chunk_len, const at::Tensor& x0,
                  const at::Tensor& mu, const at::Tensor& cond, const at::Tensor& spk, at::Tensor& out,
                  at::Tensor& workspace, bool graph) {
  TORCH_CHECK(prompt_len.size() == chunk_len.size(), "solve_packed: one prompt and chunk length per stream");
  const std::vector<int32_t> P = i32(prompt_len), T = i32(chunk_len);
  t2w_batch b{};
  b.n_streams = (int32_t)P.size();
  b.prompt_len = P.data();
  b.chunk_len = T.data();
  b.x0 = x0.data_ptr<float>();
  b.mu = mu.data_ptr<float>();
  b.cond = cond.data_ptr<float>();
  b.spk = spk.data_ptr<float>();
  b.out = out.data_ptr<float>();
  check("t2w_solve_packed", t2w_solve_packed(handle<t2w_solver>(solver), &b, workspace.data_ptr(),
                                             (size_t)workspace.numel(), graph ? T2W_FLAG_GRAPH : 0u, stream_of(out)));
}

}  // namespace

namespace {

// ---- steady state: slot pools and the caches the library keeps ----------------------------------------------------

int64_t slots_create(int64_t solver, int64_t n_slots, int64_t n_rowslots) {
  t2w_slots* p = nullptr;
  check("t2w_slots_create", t2w_slots_create(handle<t2w_solver>(solver), (int32_t)n_slots, (int32_t)n_rowslots, &p));
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(p));
}

void slots_destroy(int64_t slots) { check("t2w_slots_destroy", t2w_slots_destroy(handle<t2w_slots>(slots))); }

struct Cached {
  std::vector<int32_t> h, T;
  std::vector<uint8_t> keep;
  t2w_cached_batch b{};
};

Cached cached_batch(c10::IntArrayRef handles, c10::IntArrayRef chunk_len, c10::IntArrayRef keep, const at::Tensor& noise,
                    double temperature) {
  TORCH_CHECK(handles.size() == chunk_len.size() && handles.size() == keep.size(),
              "solve_cached: one handle, window length and keep flag per request");
  TORCH_CHECK(noise.dim() == 2 && noise.scalar_type() == at::kFloat && noise.is_contiguous(),
              "solve_cached: noise is contiguous fp32 [mel, frames]");
  Cached c;
  c.h = i32(handles);
  c.T = i32(chunk_len);
  c.keep.assign(keep.begin(), keep.end());
  c.b.n_streams = (int32_t)c.h.size();
  c.b.handle = c.h.data();
  c.b.chunk_len = c.T.data();
  c.b.keep = c.keep.data();
  c.b.noise = noise.data_ptr<float>();
  c.b.noise_frames = (int32_t)noise.size(1);
  c.b.temperature = (float)temperature;
  return c;
}

int64_t cached_workspace_bytes(int64_t solver, int64_t slots, c10::IntArrayRef handles, c10::IntArrayRef chunk_len,
                               c10::IntArrayRef keep, const at::Tensor& noise) {
  Cached c = cached_batch(handles, chunk_len, keep, noise, 1.0);
  return (int64_t)t2w_cached_workspace_bytes(handle<t2w_solver>(solver), handle<t2w_slots>(slots), &c.b);
}

void solve_cached(int64_t solver, int64_t slots, c10::IntArrayRef handles, c10::IntArrayRef chunk_len,
                  c10::IntArrayRef keep, const at::Tensor& noise, double temperature, const at::Tensor& mu,
                  const std::optional<at::Tensor>& cond, const at::Tensor& spk, at::Tensor& out, at::Tensor& workspace,
                  bool graph) {
  Cached c = cached_batch(handles, chunk_len, keep, noise, temperature);
  c.b.mu = mu.data_ptr<float>();
  c.b.cond = static_cast<const float*>(ptr(cond));
  c.b.spk = spk.data_ptr<float>();
  c.b.out = out.data_ptr<float>();
  check("t2w_solve_cached", t2w_solve_cached(handle<t2w_solver>(solver), handle<t2w_slots>(slots), &c.b,
                                             workspace.data_ptr(), (size_t)workspace.numel(),
                                             graph ? T2W_FLAG_GRAPH : 0u, stream_of(out)));
}

void solve_slots(int64_t solver, int64_t slots, c10::IntArrayRef chunk_len, c10::IntArrayRef kv_len,
                 c10::IntArrayRef kv_idx, c10::IntArrayRef cnn_rd, c10::IntArrayRef cnn_wr, const at::Tensor& x0,
                 const at::Tensor& mu, const std::optional<at::Tensor>& cond, const at::Tensor& spk, at::Tensor& out,
                 at::Tensor& workspace, bool graph) {
  const std::vector<int32_t> T = i32(chunk_len), kl = i32(kv_len), ki = i32(kv_idx), rd = i32(cnn_rd), wr = i32(cnn_wr);
  TORCH_CHECK(kl.size() == 2 * T.size() && rd.size() == kl.size() && wr.size() == kl.size(),
              "solve_slots: two key lists and conv rows (cond, uncond) per request");
  t2w_slot_batch b{};
  b.n_streams = (int32_t)T.size();
  b.chunk_len = T.data();
  b.kv_len = kl.data();
  b.kv_idx = ki.data();
  b.cnn_rd = rd.data();
  b.cnn_wr = wr.data();
  b.x0 = x0.data_ptr<float>();
  b.mu = mu.data_ptr<float>();
  b.cond = static_cast<const float*>(ptr(cond));
  b.spk = spk.data_ptr<float>();
  b.out = out.data_ptr<float>();
  const size_t need = t2w_slot_workspace_bytes(handle<t2w_solver>(solver), handle<t2w_slots>(slots), &b);
  TORCH_CHECK(need > 0, "solve_slots: invalid batch");
  TORCH_CHECK((size_t)workspace.numel() >= need, "solve_slots: workspace needs ", need, " bytes");
  check("t2w_solve_slots", t2w_solve_slots(handle<t2w_solver>(solver), handle<t2w_slots>(slots), &b,
                                           workspace.data_ptr(), (size_t)workspace.numel(),
                                           graph ? T2W_FLAG_GRAPH : 0u, stream_of(out)));
}

}  // namespace

namespace {

// ---- single kernels (the per-kernel entry points of the C ABI) -----------------------------------------------------

const uint8_t* pad_ptr(const std::optional<at::Tensor>& pad) { return static_cast<const uint8_t*>(ptr(pad)); }

void ln_mod(const at::Tensor& h, const at::Tensor& shift, const at::Tensor& scale1, double eps, at::Tensor& out,
            const std::optional<at::Tensor>& pad) {
  TORCH_CHECK(h.dim() == 2 && out.dim() == 2, "ln_mod: h [rows, C] fp32, out [rows, C] bf16");
  check("t2w_ln_mod", t2w_ln_mod(h.data_ptr<float>(), (int32_t)h.stride(0), shift.data_ptr<float>(),
                                 scale1.data_ptr<float>(), (float)eps, (int32_t)h.size(0), (int32_t)h.size(1),
                                 out.data_ptr(), (int32_t)out.stride(0), pad_ptr(pad), stream_of(h)));
}

void add_ln_mod(at::Tensor& h, const std::optional<at::Tensor>& y, const std::optional<at::Tensor>& g,
                const at::Tensor& shift, const at::Tensor& scale1, double eps, at::Tensor& out,
                const std::optional<at::Tensor>& pad) {
  TORCH_CHECK(h.dim() == 2, "add_ln_mod: h [rows, C] fp32");
  check("t2w_add_ln_mod", t2w_add_ln_mod(h.data_ptr<float>(), ptr(y), static_cast<const float*>(ptr(g)),
                                         shift.data_ptr<float>(), scale1.data_ptr<float>(), (float)eps,
                                         (int32_t)h.size(0), (int32_t)h.size(1), out.data_ptr(), pad_ptr(pad),
                                         stream_of(h)));
}

void ln_mish(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps, at::Tensor& out,
             const std::optional<at::Tensor>& pad) {
  TORCH_CHECK(x.dim() == 2, "ln_mish: x [rows, C] bf16");
  check("t2w_ln_mish", t2w_ln_mish(x.data_ptr(), w.data_ptr<float>(), b.data_ptr<float>(), (float)eps,
                                   (int32_t)x.size(0), (int32_t)x.size(1), out.data_ptr(), pad_ptr(pad), stream_of(x)));
}

void gemm(const at::Tensor& A, const at::Tensor& W, const std::optional<at::Tensor>& bias, int64_t M, int64_t N, int64_t K,
          int64_t taps, int64_t tap_row0, int64_t epi, at::Tensor& out, int64_t ldo, at::TensorList qk, double qk_eps) {
  TORCH_CHECK(A.dim() == 2, "gemm: A [rows_a, lda] bf16");
  std::vector<const float*> q;
  for (const at::Tensor& t : qk) q.push_back(t.data_ptr<float>());
  check("t2w_gemm", t2w_gemm(A.data_ptr(), (int32_t)A.size(1), (int32_t)A.size(0), W.data_ptr(),
                             static_cast<const float*>(ptr(bias)), (int32_t)M, (int32_t)N, (int32_t)K, (int32_t)taps,
                             (int32_t)tap_row0, (int32_t)epi, out.data_ptr(), (int32_t)ldo, q.empty() ? nullptr : q.data(),
                             (float)qk_eps, stream_of(A)));
}

void attn_varlen(const at::Tensor& qkv, int64_t heads, c10::IntArrayRef seq_row, c10::IntArrayRef seq_len,
                 c10::IntArrayRef prompt_len, at::Tensor& out) {
  TORCH_CHECK(seq_row.size() == seq_len.size() && seq_len.size() == prompt_len.size(),
              "attn_varlen: one row, length and prompt length per sequence");
  const std::vector<int32_t> r = i32(seq_row), l = i32(seq_len), p = i32(prompt_len);
  check("t2w_attn_varlen", t2w_attn_varlen(qkv.data_ptr(), (int32_t)qkv.size(0), (int32_t)heads, (int32_t)r.size(),
                                           r.data(), l.data(), p.data(), out.data_ptr(), stream_of(qkv)));
}

void euler_cfg(at::Tensor& x, const at::Tensor& dphi, const at::Tensor& tok_row, int64_t half_rows, double dt, double w,
               const std::optional<at::Tensor>& hx, const std::optional<at::Tensor>& out) {
  TORCH_CHECK(x.dim() == 2 && dphi.dim() == 2 && tok_row.scalar_type() == at::kInt, "euler_cfg: x [n_tok, mel], "
              "dphi [rows, ld] fp32, tok_row int32 [n_tok]");
  check("t2w_euler_cfg", t2w_euler_cfg(x.data_ptr<float>(), dphi.data_ptr<float>(), (int32_t)dphi.size(1),
                                       tok_row.data_ptr<int32_t>(), (int32_t)x.size(0), (int32_t)x.size(1),
                                       (int32_t)half_rows, (float)dt, (float)w, const_cast<void*>(ptr(hx)),
                                       hx.has_value() ? (int32_t)hx->size(1) : 0,
                                       static_cast<float*>(const_cast<void*>(ptr(out))), stream_of(x)));
}

// ---- flow encoder ---------------------------------------------------------------------------------------------------

struct Enc {
  std::vector<int32_t> h, n, tok;
  std::vector<uint8_t> fin;
  t2w_enc_batch b{};
};

Enc enc_batch(c10::IntArrayRef handles, c10::IntArrayRef n_tokens, c10::IntArrayRef final_, c10::IntArrayRef tokens) {
  TORCH_CHECK(handles.size() == n_tokens.size() && handles.size() == final_.size(),
              "encode: one handle, token count and final flag per window");
  Enc e;
  e.h = i32(handles);
  e.n = i32(n_tokens);
  e.tok = i32(tokens);
  e.fin.assign(final_.begin(), final_.end());
  e.b.n_streams = (int32_t)e.h.size();
  e.b.handle = e.h.data();
  e.b.n_tokens = e.n.data();
  e.b.final = e.fin.data();
  e.b.tokens = e.tok.data();
  return e;
}

int64_t enc_workspace_bytes(int64_t encoder, c10::IntArrayRef handles, c10::IntArrayRef n_tokens,
                            c10::IntArrayRef final_, c10::IntArrayRef tokens) {
  Enc e = enc_batch(handles, n_tokens, final_, tokens);
  return (int64_t)t2w_enc_workspace_bytes(handle<t2w_encoder>(encoder), &e.b);
}

void encode(int64_t encoder, c10::IntArrayRef handles, c10::IntArrayRef n_tokens, c10::IntArrayRef final_,
            c10::IntArrayRef tokens, at::Tensor& mu, at::Tensor& workspace, bool graph) {
  TORCH_CHECK(mu.scalar_type() == at::kFloat && mu.is_contiguous(), "encode: mu is contiguous fp32");
  Enc e = enc_batch(handles, n_tokens, final_, tokens);
  e.b.mu = mu.data_ptr<float>();
  check("t2w_encode", t2w_encode(handle<t2w_encoder>(encoder), &e.b, workspace.data_ptr(), (size_t)workspace.numel(),
                                 graph ? T2W_FLAG_GRAPH : 0u, stream_of(mu)));
}

}  // namespace

TORCH_LIBRARY(b200t2w, m) {
  m.def("create(int[] cfg_i, float[] cfg_f, float[] t_sched, Tensor[] weights, int precision) -> int", &create);
  m.def("destroy(int solver) -> ()", &destroy);
  m.def("workspace_bytes(int solver, int[] prompt_len, int[] chunk_len) -> int", &workspace_bytes);
  m.def("solve_packed(int solver, int[] prompt_len, int[] chunk_len, Tensor x0, Tensor mu, Tensor cond, Tensor spk, "
        "Tensor(a!) out, Tensor(b!) workspace, bool graph) -> ()",
        &solve_packed);
  m.def("slots_create(int solver, int n_slots, int n_rowslots) -> int", &slots_create);
  m.def("slots_destroy(int slots) -> ()", &slots_destroy);
  m.def("cached_workspace_bytes(int solver, int slots, int[] handles, int[] chunk_len, int[] keep, Tensor noise) -> int",
        &cached_workspace_bytes);
  m.def("solve_cached(int solver, int slots, int[] handles, int[] chunk_len, int[] keep, Tensor noise, "
        "float temperature, Tensor mu, Tensor? cond, Tensor spk, Tensor(a!) out, Tensor(b!) workspace, bool graph) -> ()",
        &solve_cached);
  m.def("solve_slots(int solver, int slots, int[] chunk_len, int[] kv_len, int[] kv_idx, int[] cnn_rd, int[] cnn_wr, "
        "Tensor x0, Tensor mu, Tensor? cond, Tensor spk, Tensor(a!) out, Tensor(b!) workspace, bool graph) -> ()",
        &solve_slots);
  m.def("ln_mod(Tensor h, Tensor shift, Tensor scale1, float eps, Tensor(a!) out, Tensor? pad) -> ()", &ln_mod);
  m.def("add_ln_mod(Tensor(a!) h, Tensor? y, Tensor? g, Tensor shift, Tensor scale1, float eps, Tensor(b!) out, "
        "Tensor? pad) -> ()",
        &add_ln_mod);
  m.def("ln_mish(Tensor x, Tensor w, Tensor b, float eps, Tensor(a!) out, Tensor? pad) -> ()", &ln_mish);
  m.def("gemm(Tensor A, Tensor W, Tensor? bias, int M, int N, int K, int taps, int tap_row0, int epi, Tensor(a!) out, "
        "int ldo, Tensor[] qk, float qk_eps) -> ()",
        &gemm);
  m.def("attn_varlen(Tensor qkv, int heads, int[] seq_row, int[] seq_len, int[] prompt_len, Tensor(a!) out) -> ()",
        &attn_varlen);
  m.def("euler_cfg(Tensor(a!) x, Tensor dphi, Tensor tok_row, int half_rows, float dt, float w, Tensor(b!)? hx, "
        "Tensor(c!)? out) -> ()",
        &euler_cfg);
  m.def("enc_workspace_bytes(int encoder, int[] handles, int[] n_tokens, int[] final, int[] tokens) -> int",
        &enc_workspace_bytes);
  m.def("encode(int encoder, int[] handles, int[] n_tokens, int[] final, int[] tokens, Tensor(a!) mu, "
        "Tensor(b!) workspace, bool graph) -> ()",
        &encode);
}
