// Memory-bound row kernels of the solve: LayerNorm + adaLN modulation, LayerNorm(affine) + Mish, the CFG / Euler update,
// input packing, weight conversion, and the once-per-solver time-embedding + adaLN modulation tables.
// One warp per row, 128-bit loads, warp-shuffle reductions, fp32 math (the reference's Triton kernels also normalise in
// fp32 and round once to the activation type: engine/runtime/dit_kernels.py:1-60,145-164).
#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kRowsPerBlock = 8;  // warps per block

// LN over C = 128 * V values held as V float4 per lane (column 4 (32 i + lane) + e).
template <int V>
T2W_DEV void row_stats(const float4 (&x)[V], int C, float eps, float& mean, float& rstd) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) s += (x[i].x + x[i].y) + (x[i].z + x[i].w);
  mean = warp_sum(s) / (float)C;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float a = x[i].x - mean, b = x[i].y - mean, c = x[i].z - mean, d = x[i].w - mean;
    ss += (a * a + b * b) + (c * c + d * d);
  }
  rstd = rsqrtf(warp_sum(ss) / (float)C + eps);
}

T2W_DEV void store_bf16x4(__nv_bfloat16* dst, float a, float b, float c, float d) {
  uint2 u;
  u.x = pack_bf16x2(a, b);
  u.y = pack_bf16x2(c, d);
  *reinterpret_cast<uint2*>(dst) = u;
}

// One normalised row (V float4 per lane, column 4 (32 i + lane) + e) to bf16, or to e4m3 with one power-of-two scale
// per 32-column block (a block spans 8 lanes): the e4m3 bytes go to o.out and the four scale bytes of each 128-column
// group to the row's atoms in every row-shifted layout (lane d writes layout d).
template <int V, bool E4M3>
T2W_DEV void store_row(const RowOut& o, int row, const float4 (&y)[V]) {
  const int lane = threadIdx.x & 31;
  constexpr int C = 128 * V;
  if constexpr (!E4M3) {
    __nv_bfloat16* d = static_cast<__nv_bfloat16*>(o.out) + (size_t)row * C;
#pragma unroll
    for (int i = 0; i < V; ++i) store_bf16x4(d + 4 * (32 * i + lane), y[i].x, y[i].y, y[i].z, y[i].w);
  } else {
    uint8_t* d = static_cast<uint8_t*>(o.out) + (size_t)row * C;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float a = fmaxf(fmaxf(fabsf(y[i].x), fabsf(y[i].y)), fmaxf(fabsf(y[i].z), fabsf(y[i].w)));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
      const uint32_t e = ue8m0_for_amax(a);
      const float inv = ue8m0_inv(e);
      *reinterpret_cast<uint32_t*>(d + 4 * (32 * i + lane)) = e4m3x4(y[i].x * inv, y[i].y * inv, y[i].z * inv, y[i].w * inv);
      const uint32_t word = __shfl_sync(0xffffffffu, e, 0) | (__shfl_sync(0xffffffffu, e, 8) << 8) |
                            (__shfl_sync(0xffffffffu, e, 16) << 16) | (__shfl_sync(0xffffffffu, e, 24) << 24);
      if (lane < o.n_layouts)
        *reinterpret_cast<uint32_t*>(o.sf + lane * o.layout_bytes + sf_offset(row + lane, 4 * i, C)) = word;
    }
  }
}

template <int V>
__global__ void __launch_bounds__(256) k_ln_mod(const float* __restrict__ h, int ldh, const float* __restrict__ shift,
                                                const float* __restrict__ scale1, float eps, int rows,
                                                __nv_bfloat16* __restrict__ out, int ldo,
                                                const uint8_t* __restrict__ pad) {
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int C = 128 * V;
  __nv_bfloat16* o = out + (size_t)row * ldo;
  if (pad && pad[row]) {
#pragma unroll
    for (int i = 0; i < V; ++i) store_bf16x4(o + 4 * (32 * i + lane), 0.f, 0.f, 0.f, 0.f);
    return;
  }
  float4 x[V];
  const float4* hr = reinterpret_cast<const float4*>(h + (size_t)row * ldh);
#pragma unroll
  for (int i = 0; i < V; ++i) x[i] = hr[32 * i + lane];
  float mean, rstd;
  row_stats<V>(x, C, eps, mean, rstd);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = 4 * (32 * i + lane);
    const float4 sc = __ldg(reinterpret_cast<const float4*>(scale1 + c));
    const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + c));
    store_bf16x4(o + c, fmaf((x[i].x - mean) * rstd, sc.x, sh.x), fmaf((x[i].y - mean) * rstd, sc.y, sh.y),
                 fmaf((x[i].z - mean) * rstd, sc.z, sh.z), fmaf((x[i].w - mean) * rstd, sc.w, sh.w));
  }
}

// h += g * y (the gated residual of the preceding GEMM's bf16 output y, fp32, stored back), then out = LN(h) * scale1 +
// shift (dit_kernels.py:35-60's add_ln_mod, with the residual kept in fp32).  y == nullptr: plain LN + modulation (the
// bf16 solve, whose GEMM epilogues update h themselves; with flags, the rows wait for that GEMM's tiles).
// Whether this warp's row may be read: plain programmatic ordering, or its 128-row block's GEMM tiles are complete.
// The next GEMM's weights into L2 while this kernel runs (measured at config 2: solve 30.0 -> 29.4 ms).
T2W_DEV void prefetch_next_weights(const RowWait& wt) {
  if (threadIdx.x == 0) {
    prefetch_l2_piece(wt.pf, wt.pf_bytes, blockIdx.x);
    const int n1 = (int)((wt.pf_bytes + kPrefetchPiece - 1) / kPrefetchPiece);
    if ((int)blockIdx.x >= n1) prefetch_l2_piece(wt.pf2, wt.pf2_bytes, blockIdx.x - n1);
  }
}

T2W_DEV bool row_ready(const RowWait& wt, int row) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = wait_counter(wt.flags + (row >> 7), wt.target, wt.err, wt.limit_ns);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

template <int V, bool E4M3>
__global__ void __launch_bounds__(256) k_add_ln_mod(float* __restrict__ h, const __nv_bfloat16* __restrict__ y,
                                                    const float* __restrict__ g, const float* __restrict__ shift,
                                                    const float* __restrict__ scale1, float eps, int rows, const RowOut o,
                                                    const uint8_t* __restrict__ pad, const RowWait wt) {
  // With flags the row's own GEMM tiles are awaited below instead of the whole grid.  The successor is not let in early
  // (no launch_dependents): a persistent GEMM launched early would hold whole SMs idle in its own wait while this
  // kernel's blocks still need them.
  prefetch_next_weights(wt);
  if (!wt.flags) pdl_wait();
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (wt.flags && !row_ready(wt, row)) return;
  constexpr int C = 128 * V;
  float4 x[V];
  // the fp32 residual is read and written by every add_ln_mod of the solve: kept in L2 ahead of the activations that
  // stream through it between two of them (measured: config-2 solve 30.95 -> 30.38 ms)
  float4* hr = reinterpret_cast<float4*>(h + (size_t)row * C);
  const uint64_t keep = l2_policy_evict_last();
#pragma unroll
  for (int i = 0; i < V; ++i) x[i] = ld_f4_l2hint(hr + 32 * i + lane, keep);
  if (y) {
    const uint2* yr = reinterpret_cast<const uint2*>(y + (size_t)row * C);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const uint2 u = __ldcg(yr + 32 * i + lane);  // L2: the GEMM may have written it after this SM cached lines
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + 32 * i + lane);
      x[i].x = fmaf(gg.x, a.x, x[i].x);
      x[i].y = fmaf(gg.y, a.y, x[i].y);
      x[i].z = fmaf(gg.z, c.x, x[i].z);
      x[i].w = fmaf(gg.w, c.y, x[i].w);
      st_f4_l2hint(hr + 32 * i + lane, x[i], keep);
    }
  }
  if (pad && pad[row]) {
#pragma unroll
    for (int i = 0; i < V; ++i) x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    store_row<V, E4M3>(o, row, x);
    return;
  }
  float mean, rstd;
  row_stats<V>(x, C, eps, mean, rstd);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = 4 * (32 * i + lane);
    const float4 sc = __ldg(reinterpret_cast<const float4*>(scale1 + c));
    const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + c));
    x[i] = make_float4(fmaf((x[i].x - mean) * rstd, sc.x, sh.x), fmaf((x[i].y - mean) * rstd, sc.y, sh.y),
                       fmaf((x[i].z - mean) * rstd, sc.z, sh.z), fmaf((x[i].w - mean) * rstd, sc.w, sh.w));
  }
  store_row<V, E4M3>(o, row, x);
}

template <int V, bool E4M3>
__global__ void __launch_bounds__(256) k_ln_mish(const __nv_bfloat16* __restrict__ xin, const float* __restrict__ w,
                                                 const float* __restrict__ b, float eps, int rows, const RowOut o,
                                                 const uint8_t* __restrict__ pad, const RowWait wt) {
  prefetch_next_weights(wt);
  if (!wt.flags) pdl_wait();  // no launch_dependents: see k_add_ln_mod
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (wt.flags && !row_ready(wt, row)) return;
  constexpr int C = 128 * V;
  float4 x[V];
  if (pad && pad[row]) {
#pragma unroll
    for (int i = 0; i < V; ++i) x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    store_row<V, E4M3>(o, row, x);
    return;
  }
  const uint2* xr = reinterpret_cast<const uint2*>(xin + (size_t)row * C);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint2 u = __ldcg(xr + 32 * i + lane);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    x[i] = make_float4(a.x, a.y, c.x, c.y);
  }
  float mean, rstd;
  row_stats<V>(x, C, eps, mean, rstd);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = 4 * (32 * i + lane);
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
    x[i] = make_float4(mish(fmaf((x[i].x - mean) * rstd, ww.x, bb.x)), mish(fmaf((x[i].y - mean) * rstd, ww.y, bb.y)),
                       mish(fmaf((x[i].z - mean) * rstd, ww.z, bb.z)), mish(fmaf((x[i].w - mean) * rstd, ww.w, bb.w)));
  }
  store_row<V, E4M3>(o, row, x);
}

// bf16 [rows, C] -> e4m3 with per-(row, 32-column block) power-of-two scales (the activation quantiser of the FP8
// path's test entry point; inside the solve the producing kernels quantise their own outputs).
template <int V>
__global__ void __launch_bounds__(256) k_quant_rows(const __nv_bfloat16* __restrict__ xin, int rows, const RowOut o) {
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int C = 128 * V;
  float4 x[V];
  const uint2* xr = reinterpret_cast<const uint2*>(xin + (size_t)row * C);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint2 u = xr[32 * i + lane];
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    x[i] = make_float4(a.x, a.y, c.x, c.y);
  }
  store_row<V, true>(o, row, x);
}

// Weight W [N, Kt] fp32 -> e4m3 with one power-of-two scale per 1 x 128 block, the scale repeated over the block's
// four 32-column scale slots of the atoms [Kt / 128][N / 128][512].  One warp per (row, 128-column block).
__global__ void __launch_bounds__(256) k_quant_weight(const float* __restrict__ w, int N, int Kt, uint8_t* __restrict__ w8,
                                                      uint8_t* __restrict__ sf) {
  const int item = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int kblocks = Kt / 128;
  if (item >= N * kblocks) return;
  const int n = item / kblocks, kb = item - n * kblocks;
  const float4 v = __ldg(reinterpret_cast<const float4*>(w + (size_t)n * Kt + 128 * kb) + lane);
  float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, m));
  const uint32_t e = ue8m0_for_amax(a);
  const float inv = ue8m0_inv(e);
  *reinterpret_cast<uint32_t*>(w8 + (size_t)n * Kt + 128 * kb + 4 * lane) = e4m3x4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
  if (lane == 0) {
    const int r = n & 127;
    *reinterpret_cast<uint32_t*>(sf + ((size_t)kb * (N / 128) + n / 128) * 512 + (r & 31) * 16 + (r >> 5) * 4) =
        e * 0x01010101u;
  }
}

// hx rows: [x | mu | spk | cond] for the cond half, [x | 0 | 0 | 0] for the uncond half (CFG: zeroed conditioning,
// token2wav_batch.py:672-674).  One thread per (token, mel channel).
__global__ void k_pack(const float* __restrict__ x0, const float* __restrict__ mu, const float* __restrict__ cond,
                       const float* __restrict__ spk, const int* __restrict__ tok_row, const int* __restrict__ tok_stream,
                       int n_tok, int mel, int half_rows, __nv_bfloat16* __restrict__ hx, int ld_hx,
                       float* __restrict__ x) {
  pdl_wait();
  pdl_launch();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_tok * mel) return;
  const int i = (int)(idx / mel), c = (int)(idx - (long long)i * mel);
  const int r = tok_row[i], s = tok_stream[i];
  const float xv = x0[idx];
  x[idx] = xv;
  __nv_bfloat16* a = hx + (size_t)r * ld_hx;
  __nv_bfloat16* u = hx + (size_t)(r + half_rows) * ld_hx;
  const __nv_bfloat16 xb = __float2bfloat16_rn(xv), z = __float2bfloat16_rn(0.f);
  a[c] = xb;
  a[mel + c] = __float2bfloat16_rn(mu[idx]);
  a[2 * mel + c] = __float2bfloat16_rn(spk[(size_t)s * mel + c]);
  a[3 * mel + c] = __float2bfloat16_rn(cond ? cond[idx] : 0.f);  // no condition: zeros
  u[c] = xb;
  u[mel + c] = z;
  u[2 * mel + c] = z;
  u[3 * mel + c] = z;
}

// x += dt ((1 + w) d - w u): the CFG combine and the Euler step in one pass (token2wav_batch.py:689-690).
__global__ void k_euler(float* __restrict__ x, const float* __restrict__ dphi, int ld_dphi,
                        const int* __restrict__ tok_row, int n_tok, int mel, int half_rows, float dt, float w,
                        __nv_bfloat16* __restrict__ hx, int ld_hx, float* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_tok * mel) return;
  const int i = (int)(idx / mel), c = (int)(idx - (long long)i * mel);
  const int r = tok_row[i];
  const float d = dphi[(size_t)r * ld_dphi + c], u = dphi[(size_t)(r + half_rows) * ld_dphi + c];
  const float xv = x[idx] + dt * ((1.f + w) * d - w * u);
  x[idx] = xv;
  const __nv_bfloat16 xb = __float2bfloat16_rn(xv);
  if (hx) {
    hx[(size_t)r * ld_hx + c] = xb;
    hx[(size_t)(r + half_rows) * ld_hx + c] = xb;
  }
  if (out) out[idx] = xv;
}

__global__ void k_f32_to_bf16(const float* __restrict__ s, __nv_bfloat16* __restrict__ d, long long n) {
  pdl_wait();
  pdl_launch();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) d[i] = __float2bfloat16_rn(s[i]);
}

template <class T>
__global__ void k_conv_weight(const float* __restrict__ s, T* __restrict__ d, int cout, int cin, int k) {
  pdl_wait();
  pdl_launch();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // over dst [cout, k * cin]
  if (i >= (long long)cout * cin * k) return;
  const int o = (int)(i / ((long long)k * cin));
  const int rem = (int)(i - (long long)o * k * cin);
  const int tap = rem / cin, c = rem - tap * cin;
  const float v = s[((size_t)o * cin + c) * k + tap];
  if constexpr (sizeof(T) == 2)
    d[i] = __float2bfloat16_rn(v);
  else
    d[i] = v;
}

// Time embedding: sinusoid(t * t_scale) -> Linear -> SiLU -> Linear, then SiLU (the adaLN_modulation input).  One block
// per step, one thread per hidden unit.
__global__ void k_temb(const float* __restrict__ ts, const float* __restrict__ freqs, int freq_dim, float t_scale,
                       const float* __restrict__ w1, const float* __restrict__ b1, const float* __restrict__ w2,
                       const float* __restrict__ b2, int H, float* __restrict__ silu_temb) {
  pdl_wait();
  pdl_launch();
  extern __shared__ float sm[];
  float* emb = sm;             // [freq_dim]
  float* hid = sm + freq_dim;  // [H]
  const int s = blockIdx.x;
  const float t = ts[s] * t_scale;
  const int half = freq_dim / 2;
  for (int k = threadIdx.x; k < half; k += blockDim.x) {
    const float a = t * freqs[k];
    emb[k] = cosf(a);
    emb[half + k] = sinf(a);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float acc = b1[j];
    for (int k = 0; k < freq_dim; ++k) acc = fmaf(w1[(size_t)j * freq_dim + k], emb[k], acc);
    hid[j] = acc / (1.f + expf(-acc));
  }
  __syncthreads();
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float acc = b2[j];
    for (int k = 0; k < H; ++k) acc = fmaf(w2[(size_t)j * H + k], hid[k], acc);
    silu_temb[(size_t)s * H + j] = acc / (1.f + expf(-acc));
  }
}

// Every adaLN output row j of one weight matrix W [R, H] for all steps: out[s, j] = b[j] + W[j] . silu_temb[s]; chunk
// c = j / H is a scale when (c % 3) == 1 (sh, sc, g per branch; final layer: sh, sc), stored as 1 + scale.  One warp
// per row (the row is read once for all steps), 128-bit loads.
template <int MAXS>
__global__ void k_adaln(const float* __restrict__ W, const float* __restrict__ b, int R, int H, int steps,
                        const float* __restrict__ silu_temb, float* __restrict__ out, long long step_stride,
                        int chunk_period) {
  pdl_wait();
  pdl_launch();
  extern __shared__ float st[];  // [steps, H]
  for (int i = threadIdx.x; i < steps * H; i += blockDim.x) st[i] = silu_temb[i];
  __syncthreads();
  const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (j >= R) return;
  float acc[MAXS];
#pragma unroll
  for (int s = 0; s < MAXS; ++s) acc[s] = 0.f;
  const float4* wr = reinterpret_cast<const float4*>(W + (size_t)j * H);
  for (int k4 = lane; k4 < H / 4; k4 += 32) {
    const float4 wv = __ldg(wr + k4);
#pragma unroll
    for (int s = 0; s < MAXS; ++s) {
      if (s < steps) {
        const float4 tv = *reinterpret_cast<const float4*>(st + s * H + 4 * k4);
        acc[s] = fmaf(wv.x, tv.x, fmaf(wv.y, tv.y, fmaf(wv.z, tv.z, fmaf(wv.w, tv.w, acc[s]))));
      }
    }
  }
  const int c = j / H;
  const float add = ((c % chunk_period) == 1) ? 1.f : 0.f;
#pragma unroll
  for (int s = 0; s < MAXS; ++s) {
    const float v = warp_sum(acc[s]);
    if (s < steps && lane == 0) out[s * step_stride + j] = v + b[j] + add;
  }
}

thread_local cudaError_t t_launch_err = cudaSuccess;
void check_err(cudaError_t e) {
  if (e != cudaSuccess) t_launch_err = e;
}
// Status of the launches since the last check (a launch error, else any pending CUDA error).
int check_launch() {
  cudaError_t e = t_launch_err != cudaSuccess ? t_launch_err : cudaGetLastError();
  t_launch_err = cudaSuccess;
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

unsigned blocks_for(long long n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

int launch_ln_mod(const float* h, int ldh, const float* shift, const float* scale1, float eps, int rows, int C,
                  __nv_bfloat16* out, int ldo, const uint8_t* pad, cudaStream_t st) {
  if (rows <= 0) return T2W_OK;
  if (ldh % 4 || ldo % 4) return T2W_ERR_INVALID;
  const unsigned g = blocks_for(rows, kRowsPerBlock);
  switch (C) {
    case 128: check_err(launch_k(k_ln_mod<1>, dim3(g), dim3(256), 0, st, h, ldh, shift, scale1, eps, rows, out, ldo, pad)); break;
    case 256: check_err(launch_k(k_ln_mod<2>, dim3(g), dim3(256), 0, st, h, ldh, shift, scale1, eps, rows, out, ldo, pad)); break;
    case 512: check_err(launch_k(k_ln_mod<4>, dim3(g), dim3(256), 0, st, h, ldh, shift, scale1, eps, rows, out, ldo, pad)); break;
    case 768: check_err(launch_k(k_ln_mod<6>, dim3(g), dim3(256), 0, st, h, ldh, shift, scale1, eps, rows, out, ldo, pad)); break;
    case 1024: check_err(launch_k(k_ln_mod<8>, dim3(g), dim3(256), 0, st, h, ldh, shift, scale1, eps, rows, out, ldo, pad)); break;
    default: return T2W_ERR_INVALID;
  }
  return check_launch();
}

namespace {

template <bool E4M3>
int add_ln_mod_impl(float* h, const __nv_bfloat16* y, const float* g, const float* shift, const float* scale1, float eps,
                    int rows, int C, const RowOut& o, const uint8_t* pad, cudaStream_t st, const RowWait& wt) {
  const unsigned gr = blocks_for(rows, kRowsPerBlock);
  switch (C) {
    case 128: check_err(launch_k(k_add_ln_mod<1, E4M3>, dim3(gr), dim3(256), 0, st, h, y, g, shift, scale1, eps, rows, o, pad, wt)); break;
    case 256: check_err(launch_k(k_add_ln_mod<2, E4M3>, dim3(gr), dim3(256), 0, st, h, y, g, shift, scale1, eps, rows, o, pad, wt)); break;
    case 512: check_err(launch_k(k_add_ln_mod<4, E4M3>, dim3(gr), dim3(256), 0, st, h, y, g, shift, scale1, eps, rows, o, pad, wt)); break;
    case 768: check_err(launch_k(k_add_ln_mod<6, E4M3>, dim3(gr), dim3(256), 0, st, h, y, g, shift, scale1, eps, rows, o, pad, wt)); break;
    case 1024: check_err(launch_k(k_add_ln_mod<8, E4M3>, dim3(gr), dim3(256), 0, st, h, y, g, shift, scale1, eps, rows, o, pad, wt)); break;
    default: return T2W_ERR_INVALID;
  }
  return check_launch();
}

template <bool E4M3>
int ln_mish_impl(const __nv_bfloat16* x, const float* w, const float* b, float eps, int rows, int C, const RowOut& o,
                 const uint8_t* pad, cudaStream_t st, const RowWait& wt) {
  const unsigned g = blocks_for(rows, kRowsPerBlock);
  switch (C) {
    case 128: check_err(launch_k(k_ln_mish<1, E4M3>, dim3(g), dim3(256), 0, st, x, w, b, eps, rows, o, pad, wt)); break;
    case 256: check_err(launch_k(k_ln_mish<2, E4M3>, dim3(g), dim3(256), 0, st, x, w, b, eps, rows, o, pad, wt)); break;
    case 512: check_err(launch_k(k_ln_mish<4, E4M3>, dim3(g), dim3(256), 0, st, x, w, b, eps, rows, o, pad, wt)); break;
    case 768: check_err(launch_k(k_ln_mish<6, E4M3>, dim3(g), dim3(256), 0, st, x, w, b, eps, rows, o, pad, wt)); break;
    case 1024: check_err(launch_k(k_ln_mish<8, E4M3>, dim3(g), dim3(256), 0, st, x, w, b, eps, rows, o, pad, wt)); break;
    default: return T2W_ERR_INVALID;
  }
  return check_launch();
}

bool row_out_ok(const RowOut& o) {
  if (!o.out) return false;
  if (!o.sf) return true;
  return o.n_layouts >= 1 && o.n_layouts <= 3 && (o.n_layouts == 1 || o.layout_bytes % 16 == 0) &&
         (reinterpret_cast<uintptr_t>(o.sf) & 3) == 0;
}

}  // namespace

int launch_add_ln_mod(float* h, const __nv_bfloat16* y, const float* g, const float* shift, const float* scale1, float eps,
                      int rows, int C, const RowOut& o, const uint8_t* pad, cudaStream_t st, const RowWait& wt) {
  if (rows <= 0) return T2W_OK;
  if ((y && !g) || !row_out_ok(o)) return T2W_ERR_INVALID;
  return o.sf ? add_ln_mod_impl<true>(h, y, g, shift, scale1, eps, rows, C, o, pad, st, wt)
              : add_ln_mod_impl<false>(h, y, g, shift, scale1, eps, rows, C, o, pad, st, wt);
}

int launch_ln_mish(const __nv_bfloat16* x, const float* w, const float* b, float eps, int rows, int C, const RowOut& o,
                   const uint8_t* pad, cudaStream_t st, const RowWait& wt) {
  if (rows <= 0) return T2W_OK;
  if (!row_out_ok(o)) return T2W_ERR_INVALID;
  return o.sf ? ln_mish_impl<true>(x, w, b, eps, rows, C, o, pad, st, wt)
              : ln_mish_impl<false>(x, w, b, eps, rows, C, o, pad, st, wt);
}

int launch_quant_rows(const __nv_bfloat16* x, int rows, int C, const RowOut& o, cudaStream_t st) {
  if (rows <= 0) return T2W_OK;
  if (!o.sf || !row_out_ok(o)) return T2W_ERR_INVALID;
  const unsigned g = blocks_for(rows, kRowsPerBlock);
  switch (C) {
    case 128: check_err(launch_k(k_quant_rows<1>, dim3(g), dim3(256), 0, st, x, rows, o)); break;
    case 512: check_err(launch_k(k_quant_rows<4>, dim3(g), dim3(256), 0, st, x, rows, o)); break;
    case 1536: check_err(launch_k(k_quant_rows<12>, dim3(g), dim3(256), 0, st, x, rows, o)); break;
    case 2048: check_err(launch_k(k_quant_rows<16>, dim3(g), dim3(256), 0, st, x, rows, o)); break;
    default: return T2W_ERR_INVALID;
  }
  return check_launch();
}

int launch_quant_weight(const float* w, int N, int Kt, uint8_t* w8, uint8_t* sf, cudaStream_t st) {
  if (N <= 0 || N % 128 || Kt <= 0 || Kt % 128 || !w || !w8 || !sf) return T2W_ERR_INVALID;
  const unsigned g = blocks_for(N * (Kt / 128), kRowsPerBlock);
  check_err(launch_k(k_quant_weight, dim3(g), dim3(256), 0, st, w, N, Kt, w8, sf));
  return check_launch();
}

int launch_pack(const float* x0, const float* mu, const float* cond, const float* spk, const int* tok_row,
                const int* tok_stream, int n_tok, int mel, int half_rows, __nv_bfloat16* hx, int ld_hx, float* x,
                cudaStream_t st) {
  const long long n = (long long)n_tok * mel;
  if (n <= 0) return T2W_OK;
  check_err(launch_k(k_pack, dim3(blocks_for(n, 256)), dim3(256), 0, st, x0, mu, cond, spk, tok_row, tok_stream, n_tok, mel,
                     half_rows, hx, ld_hx, x));
  return check_launch();
}

int launch_euler(float* x, const float* dphi, int ld_dphi, const int* tok_row, int n_tok, int mel, int half_rows,
                 float dt, float w, __nv_bfloat16* hx, int ld_hx, float* out, cudaStream_t st) {
  const long long n = (long long)n_tok * mel;
  if (n <= 0) return T2W_OK;
  check_err(launch_k(k_euler, dim3(blocks_for(n, 256)), dim3(256), 0, st, x, dphi, ld_dphi, tok_row, n_tok, mel, half_rows,
                     dt, w, hx, ld_hx, out));
  return check_launch();
}

int launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, long long n, cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  check_err(launch_k(k_f32_to_bf16, dim3(blocks_for(n, 256)), dim3(256), 0, st, src, dst, n));
  return check_launch();
}

int launch_conv_weight(const float* src, __nv_bfloat16* dst, int cout, int cin, int k, cudaStream_t st) {
  const long long n = (long long)cout * cin * k;
  check_err(launch_k(k_conv_weight<__nv_bfloat16>, dim3(blocks_for(n, 256)), dim3(256), 0, st, src, dst, cout, cin, k));
  return check_launch();
}

int launch_conv_weight_f32(const float* src, float* dst, int cout, int cin, int k, cudaStream_t st) {
  const long long n = (long long)cout * cin * k;
  check_err(launch_k(k_conv_weight<float>, dim3(blocks_for(n, 256)), dim3(256), 0, st, src, dst, cout, cin, k));
  return check_launch();
}

int launch_temb_mods(const float* ts, int steps, const float* freqs, int freq_dim, float t_scale, const float* fc1_w,
                     const float* fc1_b, const float* fc2_w, const float* fc2_b, int H, const float* const* ada_w,
                     const float* const* ada_b, int depth, const float* fin_w, const float* fin_b, float* silu_temb,
                     float* mods, float* final_mods, cudaStream_t st) {
  constexpr int MAXS = 16;
  if (steps > MAXS || H % 128) return T2W_ERR_UNSUPPORTED;
  check_err(launch_k(k_temb, dim3(steps), dim3(512), (freq_dim + H) * sizeof(float), st, ts, freqs, freq_dim, t_scale,
                     fc1_w, fc1_b, fc2_w, fc2_b, H, silu_temb));
  int rc = check_launch();
  if (rc) return rc;
  const size_t sm = (size_t)steps * H * sizeof(float);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_adaln<MAXS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
  }
  const int warps = 8;
  for (int b = 0; b < depth; ++b) {
    const int R = 9 * H;
    // mods layout [steps, depth, 9, H]: block b of step s at (s * depth + b) * 9H
    check_err(launch_k(k_adaln<MAXS>, dim3(blocks_for(R, warps)), dim3(32 * warps), sm, st, ada_w[b], ada_b[b], R, H,
                       steps, silu_temb, mods + (size_t)b * R, (long long)depth * R, 3));
    if ((rc = check_launch())) return rc;
  }
  check_err(launch_k(k_adaln<MAXS>, dim3(blocks_for(2 * H, warps)), dim3(32 * warps), sm, st, fin_w, fin_b, 2 * H, H, steps,
                     silu_temb, final_mods, 2LL * H, 2));
  return check_launch();
}

}  // namespace t2w
