// The HiFT vocoder (mel -> 24 kHz waveform), the step after the solve, and its C ABI (t2w_hift_*, t2w_vocode).
//
// The reference runs the third-party HiFTGenerator through its own driver functions (hift_forward_noise,
// _hift_decode, istft_overlap_add: engine/models/token2wav.py:112-245) and does the streaming bookkeeping in
// BatchedToken2Wav._vocode (engine/runtime/token2wav_batch.py:813-848): the window's mel after 8 cached frames, the
// source's first 3840 samples from the previous window, a Hamming cross-fade with the previous window's last 3840
// speech samples, and the last 3840 samples held back unless the window is final.  Here one call runs every window of
// the batch (each with its own frame count) and keeps the per-stream caches in the library.
//
// Layout: time-major fp32 rows [time, channels].  Each window is a segment at each rate (mel frames F; stage outputs at
// 8 F, 40 F and 120 F + 1 rows) with zero rows around its data so every "same" convolution reads zeros past the
// window's ends: mel rate [4 | F | 4], stage 0 [32 | 8 F | 32], stage 1 [160 | 40 F | 160], stage 2 [479 | 120 F + 1 |
// 480] (the reflection-padded row leads stage 2's data).  Every segment length at stage i is its rate times (F + 8), so
// output row u v + p of a transposed convolution's phase p lands in the next layout at a fixed offset.
//
// Precision, per the config's tf32 field: 0 strict fp32 on CUDA cores (the reference runs Token2Wav with TF32 off,
// strict_fp32, token2wav.py:44-57); 1 the reference's decode_tf32 option (all upsampling-stage parts, or the listed
// ones) on TF32 tensor cores, the f0 predictor, conv_pre and conv_post at fp32 level on the tensor cores (split form,
// or the mel rows tripled as [hi | lo | hi]); 2 every convolution at fp32 level on the tensor cores.  Tensor-core
// convolutions: tconv.cu.  CUDA-core convolutions: k_hconv, a tiled fp32 implicit-GEMM kernel (64 output rows x 64
// output channels per block, 4 x 4 per thread, 16-channel K chunks staged in shared memory) with a general row mapping
// — strided (source_downs), dilated (ResBlocks), and the polyphase form of the transposed convolutions (each output
// phase p of rate u is a convolution over the input with taps j = j0(p) + u q) — and fused epilogues: ELU (f0
// predictor), |.| (its head), Snake (the ResBlocks' second activation, applied to conv1's output), and the residual
// update x += conv2(.) that also writes the next Snake of x for the following conv1.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "tconv.h"

using namespace t2w;

namespace {

#define H_CUDA(call)                     \
  do {                                   \
    cudaError_t e_ = (call);             \
    if (e_ != cudaSuccess) {             \
      set_cuda_error(e_);                \
      return T2W_ERR_CUDA;               \
    }                                    \
  } while (0)
#define H_TRY(call)         \
  do {                      \
    int rc_ = (call);       \
    if (rc_) return rc_;    \
  } while (0)

constexpr int kMelCache = 8;          // cached mel frames (engine/models/token2wav.py:35)
constexpr int kSrcCache = 3840;       // cached source / speech samples (8 frames x 480)
constexpr int kPadMel = 4;            // zero rows on each side of a window's mel frames
constexpr int kNfft = 16, kHop = 4, kBins = kNfft / 2 + 1;
constexpr int kStftLd = 20;  // floats per STFT frame row: the 18 channels, 2 zero (rows of 80 bytes for tensor maps)
constexpr int kStftLd3 = 56;  // the tensor-core fp32 mode's tripled STFT rows: [hi 18 | lo 18 | hi 18 | 2 zero]

// ---------------------------------------------------------------- generic fp32 convolution
enum HEpi { HE_NONE = 0, HE_ELU = 1, HE_ABS = 2, HE_SNAKE = 3, HE_RESID = 4, HE_LEAKY = 5, HE_ELU_SPLIT = 6 };

struct ConvGeo {
  const int* vstart = nullptr;  // virtual rows: stream s owns [vstart[s], vstart[s + 1]), v = row - vstart[s]
  int nstreams = 0, nv = 0;     // nv = vstart[nstreams]
  const int* in_start = nullptr;  // per stream: global row of its input data, and the data's length
  const int* in_len = nullptr;
  const int* out_start = nullptr;  // per stream: global row of its output data
  const float* in = nullptr;
  int ld_in = 0, Cin = 0;
  float* out = nullptr;
  int ld_out = 0, Cout = 0;
  const float* W = nullptr;  // [Cout][taps][Cin]
  const float* bias = nullptr;
  int taps = 1, stride = 1, off = 0, dil = 1;  // input index of tap q = stride v + off + dil q (outside [0, len): 0)
  int u_out = 1, p_out = 0;                    // output index = u_out v + p_out
  int epi = HE_NONE;
  const float* alpha = nullptr;  // HE_SNAKE: this conv's Snake; HE_RESID: the next Snake (out2), per channel
  const float* inv = nullptr;    // 1 / (alpha + 1e-9)
  float* out2 = nullptr;         // HE_RESID / HE_NONE: Snake of the output for the next conv (nullptr: none)
  const float* resid = nullptr;  // HE_RESID: the residual's buffer (same layout as out; nullptr: out itself)
  float slope = 0.f;             // HE_LEAKY
};

constexpr int kTK = 16;

// The stream of virtual row r: the last s with vstart[s] <= r (vstart ascending, vstart[0] = 0 <= r < vstart[n]).
__device__ __forceinline__ int stream_of(const int* __restrict__ vstart, int n, int r) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (vstart[mid] <= r)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// fp32 rounded to the nearest TF32 value (half of the dropped unit added to the bit pattern, then the 13 low mantissa
// bits cleared); a value's split form for the tensor-core convolution is hi = tf32_rn(x), lo = tf32_rn(x - hi).
__device__ __forceinline__ float tf32_rn(float x) { return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u); }

// Snake with the sine of the tensor-core paths: the argument reduced to [-pi, pi] with 2 pi split into two floats
// (Cody-Waite), then the hardware approximation __sinf (about 2^-21 absolute there), as the convolution epilogues do.
__device__ __forceinline__ float snake_fast(float x, float a, float inv) {
  const float xa = x * a;
  const float nn = rintf(xa * 0.159154943091895336f);
  float r = fmaf(-nn, 6.28318548202514648f, xa);
  r = fmaf(-nn, -1.74845553146951715e-07f, r);
  const float sv = __sinf(r);
  return x + inv * (sv * sv);
}

__device__ __forceinline__ float snake(float x, float a, float inv) {
  const float s = sinf(x * a);
  return x + inv * (s * s);
}

// TM x TN outputs per block, 256 threads of 4 x 4; K = taps * Cin flattened (tap-major), 16 per shared-memory chunk, so
// narrow inputs (18 STFT channels, 80 mel channels) waste no chunk lanes.
template <int TM, int TN>
__global__ void __launch_bounds__(256) k_hconv(const ConvGeo g) {
  constexpr int TX = TN / 4;  // threads across columns
  __shared__ float As[kTK][TM + 4];
  __shared__ float Ws[kTK][TN + 4];
  __shared__ int rowb[TM];  // per tile row: global input row of the stream's data start, or -1
  __shared__ int rowv[TM];  // input index of tap 0
  __shared__ int rowl[TM];  // the stream's input data length
  __shared__ int rowo[TM];  // output row, or -1 past the last virtual row
  pdl_wait();
  pdl_launch();
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * TM, c0 = blockIdx.y * TN;
  for (int t = tid; t < TM; t += 256) {
    const int r = r0 + t;
    if (r < g.nv) {
      const int s = stream_of(g.vstart, g.nstreams, r), v = r - g.vstart[s];
      rowb[t] = g.in_start[s];
      rowv[t] = g.stride * v + g.off;
      rowl[t] = g.in_len[s];
      rowo[t] = g.out_start[s] + g.u_out * v + g.p_out;
    } else {
      rowb[t] = -1;
      rowv[t] = 0;
      rowl[t] = 0;
      rowo[t] = -1;
    }
  }
  __syncthreads();
  const int ty = tid / TX, tx = tid % TX;
  float acc[4][4] = {};
  const int K = g.taps * g.Cin;
  for (int k0 = 0; k0 < K; k0 += kTK) {
    // A: TM rows x 16 of K
    for (int i = tid; i < TM * kTK; i += 256) {
      const int rr = i / kTK, kk = i % kTK, k = k0 + kk;
      float v = 0.f;
      if (k < K && rowb[rr] >= 0) {
        const int q = k / g.Cin, ci = k - q * g.Cin;
        const int idx = rowv[rr] + g.dil * q;
        if (idx >= 0 && idx < rowl[rr]) v = g.in[(size_t)(rowb[rr] + idx) * g.ld_in + ci];
      }
      As[kk][rr] = v;
    }
    // W: TN output channels x 16 of K
    for (int i = tid; i < TN * kTK; i += 256) {
      const int oo = i / kTK, kk = i % kTK, k = k0 + kk, co = c0 + oo;
      Ws[kk][oo] = (co < g.Cout && k < K) ? g.W[(size_t)co * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kTK; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      const float4 w = *reinterpret_cast<const float4*>(&Ws[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (r0 + ty * 4 + i >= g.nv) continue;
    const size_t orow = (size_t)rowo[ty * 4 + i];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int co = c0 + tx * 4 + j;
      if (co >= g.Cout) continue;
      float y = acc[i][j] + g.bias[co];
      float* dst = g.out + orow * g.ld_out + co;
      switch (g.epi) {
        case HE_ELU: y = y > 0.f ? y : expm1f(y); break;
        case HE_ELU_SPLIT: {  // [hi | lo] of the ELU output (ld_out = 2 Cout) for a split-form tensor-core conv
          y = y > 0.f ? y : expm1f(y);
          const float hi = tf32_rn(y);
          dst[g.Cout] = tf32_rn(y - hi);
          y = hi;
          break;
        }
        case HE_ABS: y = fabsf(y); break;
        case HE_SNAKE: y = snake(y, g.alpha[co], g.inv[co]); break;
        case HE_LEAKY: y = y > 0.f ? y : y * g.slope; break;
        case HE_RESID: {
          y = y + (g.resid ? g.resid[orow * g.ld_out + co] : *dst);
          if (g.out2) g.out2[orow * g.ld_out + co] = snake(y, g.alpha[co], g.inv[co]);
          break;
        }
        default:
          if (g.out2) g.out2[orow * g.ld_out + co] = snake(y, g.alpha[co], g.inv[co]);
          break;
      }
      *dst = y;
    }
  }
}

// ---------------------------------------------------------------- elementwise / layout kernels
// The window's mel rows: [cached 8 frames (unless first) | window frames] into the mel-rate layout (token-major input).
struct HRow {
  int F, first, cache, mel_off;   // mel frames (with the cached ones), first window, cache row, window's input row
  int mel0, s0, s1, s2;           // data start rows at the mel rate and the three stage rates
  int smp0;                        // first sample of the window in the sample-rate arrays
  int last;                        // final window
  int out0, out_len;               // output samples: offset and count
};

// mel3 (may be null): the rows tripled as [hi | lo | hi] (3 C floats a row), the input of the tensor-core convs.
__global__ void k_mel_in(const float* __restrict__ win_mel, const HRow* __restrict__ rows, const float* __restrict__ cache,
                         int cache_ld, int C, float* __restrict__ mel, float* __restrict__ mel3) {
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.y];
  const int t = blockIdx.x;
  if (t >= e.F) return;
  const int nc = e.first ? 0 : kMelCache;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float v = t < nc ? cache[(size_t)e.cache * cache_ld + t * C + c] : win_mel[(size_t)(e.mel_off + t - nc) * C + c];
    mel[(size_t)(e.mel0 + t) * C + c] = v;
    if (mel3) {
      float* r = mel3 + (size_t)(e.mel0 + t) * 3 * C;
      const float hi = tf32_rn(v);
      r[c] = hi;
      r[C + c] = tf32_rn(v - hi);
      r[2 * C + c] = hi;
    }
  }
}

// x_j = x + src (three copies for the three ResBlocks), and Snake_j(x_j) of each ResBlock's first activation.
struct Snake3 {
  const float *al[3], *inv[3];
};
// xb = ups(x) + source branch (every row), the three ResBlocks' first Snakes of it; each ResBlock's first residual
// update reads xb and writes its own stream, so xb is not copied three times.  Four consecutive channels per thread
// (C % 4 == 0).  split: the Snakes as [hi | lo] rows of 2 C floats (the split-form convs' input).  fast: the Snakes'
// sine as on the tensor-core paths (snake_fast), else sinf.
__global__ void k_fanout(const float* x, const float* __restrict__ src, long long n, int C, int split, int fast,
                         float* xb, float* a0, float* a1, float* a2, const Snake3 sn) {
  pdl_wait();
  pdl_launch();
  const long long n4 = n >> 2;
  for (long long i4 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i4 < n4; i4 += (long long)gridDim.x * blockDim.x) {
    const long long i = i4 << 2, r = i / C;
    const int c = (int)(i - r * C);
    const float4 xv = reinterpret_cast<const float4*>(x)[i4], sv = reinterpret_cast<const float4*>(src)[i4];
    const float v[4] = {xv.x + sv.x, xv.y + sv.y, xv.z + sv.z, xv.w + sv.w};
    reinterpret_cast<float4*>(xb)[i4] = make_float4(v[0], v[1], v[2], v[3]);
    float* const a[3] = {a0, a1, a2};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float4 al = *reinterpret_cast<const float4*>(sn.al[k] + c);
      const float4 iv = *reinterpret_cast<const float4*>(sn.inv[k] + c);
      const float alv[4] = {al.x, al.y, al.z, al.w}, ivv[4] = {iv.x, iv.y, iv.z, iv.w};
      float y[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) y[q] = fast ? snake_fast(v[q], alv[q], ivv[q]) : snake(v[q], alv[q], ivv[q]);
      if (split) {
        float hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          hi[q] = tf32_rn(y[q]);
          lo[q] = tf32_rn(y[q] - hi[q]);
        }
        *reinterpret_cast<float4*>(a[k] + r * 2 * C + c) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4*>(a[k] + r * 2 * C + C + c) = make_float4(lo[0], lo[1], lo[2], lo[3]);
      } else {
        *reinterpret_cast<float4*>(a[k] + i) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
  }
}

// y = leaky_relu((x0 + x1 + x2) / 3, slope), four consecutive channels per thread (C % 4 == 0).
// split: y holds [hi | lo] rows of 2 C floats (the input of a split-form tensor-core conv), else C floats per row.
__global__ void k_avg3(const float* __restrict__ x0, const float* __restrict__ x1, const float* __restrict__ x2,
                       long long n, int C, int split, float slope, float* __restrict__ y) {
  pdl_wait();
  pdl_launch();
  const long long n4 = n >> 2;
  for (long long i4 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i4 < n4; i4 += (long long)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x0)[i4], b = reinterpret_cast<const float4*>(x1)[i4],
                 c3 = reinterpret_cast<const float4*>(x2)[i4];
    float v[4] = {((a.x + b.x) + c3.x) / 3.f, ((a.y + b.y) + c3.y) / 3.f, ((a.z + b.z) + c3.z) / 3.f,
                  ((a.w + b.w) + c3.w) / 3.f};
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = v[q] > 0.f ? v[q] : v[q] * slope;
    if (split) {
      const long long i = i4 << 2, r = i / C, c = i - r * C;
      float hi[4], lo[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        hi[q] = tf32_rn(v[q]);
        lo[q] = tf32_rn(v[q] - hi[q]);
      }
      *reinterpret_cast<float4*>(y + r * 2 * C + c) = make_float4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<float4*>(y + r * 2 * C + C + c) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    } else {
      reinterpret_cast<float4*>(y)[i4] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

// The f0 predictor's head, |w . x + b| per data row of the mel-rate layout (one warp per row; padding rows skipped).
__global__ void k_f0_head(const float* __restrict__ x, int ld, int C, const float* __restrict__ w,
                          const float* __restrict__ b, const uint8_t* __restrict__ pad, int rows, float* __restrict__ f0) {
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows || pad[r]) return;
  float acc = 0.f;
  for (int c = lane; c < C; c += 32) acc = fmaf(x[(size_t)r * ld + c], w[c], acc);
  acc = warp_sum(acc);
  if (lane == 0) f0[r] = fabsf(acc + b[0]);
}

// Stage 2's reflection pad: the row before the transposed conv's output = its second row.
__global__ void k_reflect_row(float* __restrict__ x, const HRow* __restrict__ rows, int C) {
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.x];
  for (int c = threadIdx.x; c < C; c += blockDim.x) x[(size_t)e.s2 * C + c] = x[(size_t)(e.s2 + 2) * C + c];
}

// The harmonic source, per window: rad of frame k and harmonic h = frac(f0_k (h + 1) / sr); its cumulative phase over
// frames (2 pi sum), interpolated linearly to samples after the x upsample_scale product (the reference's
// F.interpolate(... * upsample_scale, scale_factor=upsample_scale, mode="linear")); the sine, voiced / unvoiced noise
// mix, linear over harmonics, tanh.  Grid (sample chunks of kSrcChunk, windows): every block of a window rebuilds the
// window's frame phases in shared memory (F sequential steps per harmonic) and writes its chunk of samples.
constexpr int kMaxFrames = 512;
constexpr int kMaxHarm = 16;
constexpr int kSrcChunk = 1024;
__global__ void __launch_bounds__(256) k_source(const float* __restrict__ f0, const HRow* __restrict__ rows,
                                               const float* __restrict__ noise, const float* __restrict__ lin_w,
                                               float lin_b, int dim, float sr, float upscale, float sine_amp,
                                               float noise_std, float vthr, const float* __restrict__ cache,
                                               int cache_ld, int cache_src_off, float* __restrict__ src) {
  __shared__ float ph[kMaxFrames * kMaxHarm];
  __shared__ float f0s[kMaxFrames];
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.y];
  const int F = e.F;
  const int N = F * (int)upscale;
  const int n0 = blockIdx.x * kSrcChunk;
  if (n0 >= N) return;
  const bool cached = !e.first;
  if (cached && n0 + kSrcChunk <= kSrcCache) {  // the whole chunk comes from the cached source tail
    for (int n = n0 + threadIdx.x; n < n0 + kSrcChunk; n += blockDim.x)
      src[e.smp0 + n] = cache[(size_t)e.cache * cache_ld + cache_src_off + n];
    return;
  }
  for (int t = threadIdx.x; t < F; t += blockDim.x) f0s[t] = f0[e.mel0 + t];
  __syncthreads();
  // cumulative phase per harmonic (sequential over frames, one thread per harmonic)
  if (threadIdx.x < dim) {
    const int h = threadIdx.x;
    float c = 0.f;
    for (int t = 0; t < F; ++t) {
      const float fn = f0s[t] * (float)(h + 1);
      const float r = fn / sr;
      c += r - floorf(r);
      ph[t * dim + h] = (c * 2.f) * 3.14159265358979323846f * upscale;
    }
  }
  __syncthreads();
  const float scale = 1.f / upscale;
  const int n1 = min(N, n0 + kSrcChunk);
  for (int n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
    float out;
    if (cached && n < kSrcCache) {
      out = cache[(size_t)e.cache * cache_ld + cache_src_off + n];
    } else {
      float sx = scale * ((float)n + 0.5f) - 0.5f;
      if (sx < 0.f) sx = 0.f;
      const int i0 = (int)sx;
      const int i1 = i0 + (i0 < F - 1 ? 1 : 0);
      const float l1 = sx - (float)i0, l0 = 1.f - l1;
      const float f = f0s[n / (int)upscale];
      const float uv = (f > vthr) ? 1.f : 0.f;
      const float namp = uv * noise_std + (1.f - uv) * sine_amp / 3.f;
      float acc = lin_b;
      for (int h = 0; h < dim; ++h) {
        const float phase = l0 * ph[i0 * dim + h] + l1 * ph[i1 * dim + h];
        const float sine = sinf(phase) * sine_amp * uv + namp * noise[(size_t)e.smp0 * dim + (size_t)h * N + n];
        acc = fmaf(lin_w[h], sine, acc);
      }
      out = tanhf(acc);
    }
    src[e.smp0 + n] = out;
  }
}

// STFT of the source (n_fft 16, hop 4, periodic Hann, center with reflect padding): frame t of the window into stage-2
// row s2 + t, 9 real parts then 9 imaginary parts.
// x3: the frame row tripled as [hi 18 | lo 18 | hi 18] (the tensor-core fp32 mode's source_down input).
__global__ void k_stft(const float* __restrict__ src, const HRow* __restrict__ rows, const float* __restrict__ tw,
                       float* __restrict__ out, int ld_out, float upscale, int x3) {
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.y];
  const int N = e.F * (int)upscale;
  const int frames = N / kHop + 1;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= frames) return;
  float x[kNfft];
#pragma unroll
  for (int k = 0; k < kNfft; ++k) {
    int j = kHop * t + k - kNfft / 2;
    if (j < 0) j = -j;
    if (j >= N) j = 2 * (N - 1) - j;
    x[k] = src[e.smp0 + j] * tw[k];  // tw[0..15]: the window
  }
  float* o = out + (size_t)(e.s2 + t) * ld_out;
#pragma unroll
  for (int m = 0; m < kBins; ++m) {
    float re = 0.f, im = 0.f;
#pragma unroll
    for (int k = 0; k < kNfft; ++k) {
      re = fmaf(x[k], tw[16 + ((m * k) & 15)], re);   // cos(2 pi m k / 16)
      im = fmaf(-x[k], tw[32 + ((m * k) & 15)], im);  // -sin(2 pi m k / 16)
    }
    if (x3) {
      const float hr = tf32_rn(re), hm = tf32_rn(im);
      o[m] = hr;
      o[kBins + m] = hm;
      o[2 * kBins + m] = tf32_rn(re - hr);
      o[3 * kBins + m] = tf32_rn(im - hm);
      o[4 * kBins + m] = hr;
      o[5 * kBins + m] = hm;
    } else {
      o[m] = re;
      o[kBins + m] = im;
    }
  }
}

// magnitude / phase of conv_post's output -> inverse STFT (per-frame real inverse DFT, window, overlap-add, / the
// summed squared window, centre trim), clamp; then the cross-fade with the previous window's speech, the caches and the
// window's output samples.  A block per 1024 output samples: the bins of the frames they overlap once (exp, sin, the
// complex value: 4 transcendentals per frame and bin rather than per sample), then the frames' inverse DFT values, then
// the overlap-add per sample, every sum in the order of the per-sample form.
constexpr int kIstftChunk = 1024;                                // output samples per block
constexpr int kIstftFrames = (kIstftChunk + kNfft) / kHop + 2;     // frames a chunk's samples overlap, at most
__global__ void __launch_bounds__(256) k_istft_out(const float* __restrict__ y, int ld_y, const HRow* __restrict__ rows,
                                                   const float* __restrict__ tw, const double* __restrict__ hamming,
                                                   float audio_limit, float upscale, float* __restrict__ speech,
                                                   const float* __restrict__ cache, int cache_ld, int cache_sp_off,
                                                   float* __restrict__ out) {
  __shared__ float spec[kIstftFrames][2 * kBins];  // the chunk's frames: bins as re, im
  __shared__ float fv[kIstftFrames][kNfft];        // the frames' inverse DFT values (before the window)
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.y];
  const int N = e.F * (int)upscale;
  const int n0 = blockIdx.x * kIstftChunk;
  if (n0 >= N) return;
  const int n1 = min(N, n0 + kIstftChunk);
  const int T = N / kHop + 1;
  // frames t with 0 <= j - hop t < n_fft for some j = n + n_fft / 2 of the chunk
  const int t_lo = max(0, (n0 + kNfft / 2 - kNfft + kHop) / kHop), t_hi = min(T - 1, (n1 - 1 + kNfft / 2) / kHop);
  const int nf = t_hi - t_lo + 1;
  // 1. each frame's bins once: magnitude exp (clipped at 100), phase sin, the complex value
  for (int i = threadIdx.x; i < nf * kBins; i += blockDim.x) {
    const int tt = i / kBins, m = i - tt * kBins;
    const float* row = y + (size_t)(e.s2 + t_lo + tt) * ld_y;
    const float mag = fminf(expf(row[m]), 100.f);
    const float ph = sinf(row[kBins + m]);
    spec[tt][m] = mag * cosf(ph);
    spec[tt][kBins + m] = mag * sinf(ph);
  }
  __syncthreads();
  // 2. each frame's real inverse DFT at its 16 positions
  for (int i = threadIdx.x; i < nf * kNfft; i += blockDim.x) {
    const int tt = i / kNfft, k = i - tt * kNfft;
    float v = 0.f;
#pragma unroll
    for (int m = 0; m < kBins; ++m) {
      const float re = spec[tt][m], im = spec[tt][kBins + m];
      const float c = tw[16 + ((m * k) & 15)], sn = tw[32 + ((m * k) & 15)];
      const float term = re * c - im * sn;
      v += (m == 0 || m == kBins - 1) ? ((m == 0) ? re : re * c) : 2.f * term;
    }
    fv[tt][k] = v * (1.f / kNfft);
  }
  __syncthreads();
  // 3. per sample: overlap-add of its frames through the window, / the summed squared window, clamp
  for (int n = n0 + threadIdx.x; n < n1; n += blockDim.x) {
    const int j = n + kNfft / 2;  // position in the overlap-added signal
    float acc = 0.f, env = 0.f;
    for (int t = max(0, (j - kNfft + kHop) / kHop); t <= j / kHop && t < T; ++t) {
      const int k = j - kHop * t;
      if (k < 0 || k >= kNfft) continue;
      acc = fmaf(fv[t - t_lo][k], tw[k], acc);
      env = fmaf(tw[k], tw[k], env);
    }
    float sp = fminf(fmaxf(acc / env, -audio_limit), audio_limit);
    const float* cache_row = cache + (size_t)e.cache * cache_ld;
    if (!e.first && n < kSrcCache)  // cross-fade with the previous window's last speech samples (float64 window)
      sp = (float)((double)sp * hamming[n] + (double)cache_row[cache_sp_off + n] * hamming[kSrcCache + n]);
    speech[e.smp0 + n] = sp;
    // output: held back tail (unless final), leading silence of a first window
    if (e.last) {
      out[e.out0 + n] = sp;
    } else if (e.first) {
      if (n + kSrcCache < N) out[e.out0 + kSrcCache + n] = sp;
      if (n < kSrcCache) out[e.out0 + n] = 0.f;
    } else if (n < N - kSrcCache) {
      out[e.out0 + n] = sp;
    }
  }
}

// The caches after a window (after k_istft_out has written the speech): the last 8 mel frames, 3840 source and 3840
// speech samples.  One block per window.
__global__ void k_hift_caches(const HRow* __restrict__ rows, const float* __restrict__ mel, int C,
                              const float* __restrict__ src, const float* __restrict__ speech, float* __restrict__ cache,
                              int cache_ld, int mel_off, int src_off, int sp_off, float upscale) {
  pdl_wait();
  pdl_launch();
  const HRow e = rows[blockIdx.x];
  const int N = e.F * (int)upscale;
  float* c = cache + (size_t)e.cache * cache_ld;
  for (int i = threadIdx.x; i < kMelCache * C; i += blockDim.x) {
    const int t = e.F - kMelCache + i / C;
    c[mel_off + i] = t >= 0 ? mel[(size_t)(e.mel0 + t) * C + i % C] : 0.f;
  }
  for (int i = threadIdx.x; i < kSrcCache; i += blockDim.x) {
    const int n = N - kSrcCache + i;
    c[src_off + i] = n >= 0 ? src[e.smp0 + n] : 0.f;
    c[sp_off + i] = n >= 0 ? speech[e.smp0 + n] : 0.f;
  }
}

inline int ck(cudaError_t e) {
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

int grid_for(long long n) {
  const long long b = (n + 255) / 256;
  return (int)std::min<long long>(b, 148ll * 16);
}

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

// ---------------------------------------------------------------- runtime

struct HConv {
  float* W = nullptr;  // [Cout][taps][Cin]
  float* b = nullptr;
  int Cin = 0, Cout = 0, k = 0;
  float* Ws = nullptr;  // split form [Cout][k][W_hi | W_lo | W_hi] (the tensor-core fp32 mode)
};
struct HRes {
  HConv c1[3], c2[3];
  float *a1 = nullptr, *i1 = nullptr, *a2 = nullptr, *i2 = nullptr;  // [3][C] alphas and 1 / (alpha + 1e-9)
  int k = 0;
};
struct HStage {
  int u = 0, k = 0, pad = 0, Cin = 0, Cout = 0;
  std::vector<HConv> phase;  // polyphase weights of the transposed conv: phase p -> [Cout][nq][Cin]
  std::vector<int> nq, c;    // taps and input offset of each phase
  float* b = nullptr;
  HConv down;
  int down_stride = 1, down_pad = 0;
  // source_down on the tensor cores: a 3-tap conv over the STFT rows grouped by the stride (space to depth, S frames of
  // kStftLd floats per group row); weights [Cout][taps][roundup(S kStftLd, 32)]
  float* down_tc = nullptr;
  int down_taps = 0, down_q0 = 0;
  float* down_x3 = nullptr;  // the same over tripled STFT rows [hi | lo | hi] (the tensor-core fp32 mode)
  HRes src, res[3];
};

struct t2w_hift {
  t2w_hift_config cfg{};
  int device = 0, n_streams = 0, max_frames = 0;
  std::vector<void*> allocs;
  HConv f0c[8], f0head, pre, post;
  int f0_layers = 0;
  // split-form (3xTF32) weights [Cout][taps][W_hi | W_lo | W_hi] of the f0 layers after the first and of conv_post
  // (its 18 outputs padded to 32), for the tensor-core convolution where the reference keeps fp32
  float* f0s[8] = {};
  float* post_ws = nullptr;
  float* post_bs = nullptr;
  int f0_tc = 0, post_tc = 0;  // those layers run on the tensor cores
  // conv_pre and the first f0 layer over the mel rows tripled [hi | lo | hi] (80 channels: no split form), weights
  // [Cout][k][W_hi | W_hi | W_lo, padded to a multiple of 32]: fp32-level products on the tensor cores
  float *pre_x3 = nullptr, *f00_x3 = nullptr;
  int x3 = 0;  // every convolution on the tensor cores in split form (3xTF32, fp32-level): tf32 = 2
  float* lin_w = nullptr;
  float lin_b = 0.f;
  HStage st[3];
  float* tw = nullptr;        // window, cos and sin tables (48 floats)
  double* hamming = nullptr;  // 7680
  float* cache = nullptr;     // [n_streams][8 mel frames x C | 3840 source | 3840 speech]
  int cache_ld = 0;
  int tf32 = 0;               // some upsampling-stage part on the TF32 tensor-core convolution
  uint32_t tc_parts = 0;      // those parts: bit 3 s + p (p 0 transposed conv, 1 source branch, 2 ResBlocks)
  int* err = nullptr;         // bounded-wait error word of the tensor-core kernels
  std::vector<int> row_free;
  std::vector<uint8_t> row_live, row_first;
  std::mutex mu;
  // pinned host images of the calls' plans, rotated between uploads (a copy from pageable memory would first
  // synchronise the stream, so the host could not plan a call while the previous one runs)
  static constexpr int kStaging = 2;
  struct Staging {
    void* host = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;
    bool used = false;
  };
  Staging staging[kStaging];
  int staging_next = 0;
  // the calls' scratch: a stream-ordered pool of this vocoder's own that keeps its memory reserved between calls (the
  // default pool hands freed memory back at the next synchronisation, and remapping it costs every call milliseconds)
  cudaMemPool_t pool = nullptr;
  // CUDA graphs of whole calls (T2W_FLAG_GRAPH), one per launch structure (the call's sizes), captured the second time
  // a structure is seen; each owns the workspace its launches address
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    uint8_t* ws = nullptr;
    cudaEvent_t done = nullptr;  // recorded after its latest launch
  };
  std::unordered_map<uint64_t, Graph> graphs;
  std::unordered_map<uint64_t, int> seen;
  cudaStream_t cap_stream = nullptr;
  int64_t n_replays = 0, n_captures = 0, n_eager = 0;
  // a call's f0 predictor, harmonic source and STFT run on `side`, beside conv_pre and stage 0's transposed conv
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  // every stage: ResBlocks 1 and 2 on streams of their own, beside ResBlock 0
  cudaStream_t res_st[2] = {nullptr, nullptr};
  cudaEvent_t res_ev[2] = {nullptr, nullptr};
};

namespace {

template <class T>
int halloc(t2w_hift* h, T** p, size_t n) {
  void* q = nullptr;
  const cudaError_t rc = cudaMalloc(&q, std::max<size_t>(n * sizeof(T), 16));
  if (rc != cudaSuccess) {
    set_cuda_error(rc);
    return rc == cudaErrorMemoryAllocation ? T2W_ERR_OOM : T2W_ERR_CUDA;
  }
  h->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return T2W_OK;
}
int up(t2w_hift* h, const std::vector<float>& v, float** dst) {
  H_TRY(halloc(h, dst, v.size()));
  H_CUDA(cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return T2W_OK;
}
int down(const float* src, size_t n, std::vector<float>& out) {
  out.resize(n);
  H_CUDA(cudaMemcpy(out.data(), src, n * 4, cudaMemcpyDeviceToHost));
  return T2W_OK;
}
// Conv1d weight [out, in, k] -> [out][k][in] (tap-major rows per output channel).
int conv(t2w_hift* h, const float* w, const float* b, int Cout, int Cin, int k, HConv* c) {
  std::vector<float> hw, hb, t((size_t)Cout * k * Cin);
  H_TRY(down(w, (size_t)Cout * Cin * k, hw));
  H_TRY(down(b, Cout, hb));
  for (int o = 0; o < Cout; ++o)
    for (int i = 0; i < Cin; ++i)
      for (int j = 0; j < k; ++j) t[((size_t)o * k + j) * Cin + i] = hw[((size_t)o * Cin + i) * k + j];
  c->Cin = Cin;
  c->Cout = Cout;
  c->k = k;
  H_TRY(up(h, t, &c->W));
  return up(h, hb, &c->b);
}
// fp32 -> nearest TF32 value (the device tf32_rn, on the host).
float tf32_rn_host(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  u = (u + 0x1000u) & 0xFFFFE000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// Split-form weights of a [Cout][k][Cin] conv for the tensor-core convolution: [n_pad][k][W_hi | W_lo | W_hi] (W_hi
// the weight rounded to TF32, W_lo the remainder rounded to TF32; rows past Cout zero) and the bias padded to n_pad
// (b == nullptr: the layer keeps its own bias).
int split_weights(t2w_hift* h, const HConv& cv, int n_pad, float** W, float** b) {
  std::vector<float> w, bb;
  H_TRY(down(cv.W, (size_t)cv.Cout * cv.k * cv.Cin, w));
  H_TRY(down(cv.b, cv.Cout, bb));
  std::vector<float> t((size_t)n_pad * cv.k * 3 * cv.Cin, 0.f), tb(n_pad, 0.f);
  for (int o = 0; o < cv.Cout; ++o) {
    tb[o] = bb[o];
    for (int j = 0; j < cv.k; ++j) {
      float* d = &t[((size_t)o * cv.k + j) * 3 * cv.Cin];
      for (int i = 0; i < cv.Cin; ++i) {
        const float x = w[((size_t)o * cv.k + j) * cv.Cin + i];
        const float hi = tf32_rn_host(x);
        d[i] = hi;
        d[cv.Cin + i] = tf32_rn_host(x - hi);
        d[2 * cv.Cin + i] = hi;
      }
    }
  }
  H_TRY(up(h, t, W));
  return b ? up(h, tb, b) : T2W_OK;
}

// source_down of stage s as a conv over the STFT rows grouped by its stride S.  The call layout puts stage s's output
// row R (R = e.s_s + v, make_plan) over STFT row S R + delta + v-relative taps: e.s2 = S e.s_s - 1 for stages 0 and 1
// (delta = -1), e.s2 = e.s_2 for stage 2 (delta = 0).  Output v reads frames S v + t - pad (t < k), i.e. rows
// S R + d + t with d = delta - pad, which are group row R + q, frame j of it, for S q + j = d + t: taps q from
// floor(d / S) to floor((d + k - 1) / S), weight [o][q - q0][j kStftLd + c] = W[o][c][S q + j - d].
// x3: over the tripled STFT rows (kStftLd3 floats a frame), the frame's weights [W_hi | W_hi | W_lo].
int grouped_down(t2w_hift* h, HStage& g, int s, bool x3 = false) {
  const int S = g.down_stride, k = g.down.k, Cin = g.down.Cin, Cout = g.down.Cout;
  const int d = (s == 2 ? 0 : -1) - g.down_pad;
  auto fdiv = [](int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); };
  const int q0 = fdiv(d, S), q1 = fdiv(d + k - 1, S), taps = q1 - q0 + 1;
  const int ld = x3 ? kStftLd3 : kStftLd;
  const int cg = S * ld, cp = (cg + 31) / 32 * 32;
  std::vector<float> w;
  H_TRY(down(g.down.W, (size_t)Cout * k * Cin, w));  // [o][t][c]
  std::vector<float> t((size_t)Cout * taps * cp, 0.f);
  for (int o = 0; o < Cout; ++o)
    for (int qi = 0; qi < taps; ++qi)
      for (int j = 0; j < S; ++j) {
        const int tap = S * (q0 + qi) + j - d;
        if (tap < 0 || tap >= k) continue;
        for (int c = 0; c < Cin; ++c) {
          const float x = w[((size_t)o * k + tap) * Cin + c];
          float* dd = &t[((size_t)o * taps + qi) * cp + j * ld];
          if (x3) {
            const float hi = tf32_rn_host(x);
            dd[c] = hi;
            dd[Cin + c] = hi;
            dd[2 * Cin + c] = tf32_rn_host(x - hi);
          } else {
            dd[c] = x;
          }
        }
      }
  g.down_taps = taps;
  g.down_q0 = q0;
  return up(h, t, x3 ? &g.down_x3 : &g.down_tc);
}

// Weights of a [Cout][k][Cin] conv over rows tripled as [hi | lo | hi] (ld = 3 Cin floats): per tap [W_hi | W_hi |
// W_lo], padded to a multiple of 32 columns, so a plain TF32 conv over the tripled rows sums hi W_hi + lo W_hi +
// hi W_lo.
int x3_weights(t2w_hift* h, const HConv& cv, float** W) {
  std::vector<float> w;
  H_TRY(down(cv.W, (size_t)cv.Cout * cv.k * cv.Cin, w));
  const int cp = (3 * cv.Cin + 31) / 32 * 32;
  std::vector<float> t((size_t)cv.Cout * cv.k * cp, 0.f);
  for (int o = 0; o < cv.Cout; ++o)
    for (int j = 0; j < cv.k; ++j) {
      float* d = &t[((size_t)o * cv.k + j) * cp];
      for (int i = 0; i < cv.Cin; ++i) {
        const float x = w[((size_t)o * cv.k + j) * cv.Cin + i];
        const float hi = tf32_rn_host(x);
        d[i] = hi;
        d[cv.Cin + i] = hi;
        d[2 * cv.Cin + i] = tf32_rn_host(x - hi);
      }
    }
  return up(h, t, W);
}

int snake_params(t2w_hift* h, const float* const* a, int C, float** al, float** inv) {
  std::vector<float> va((size_t)3 * C), vi((size_t)3 * C);
  for (int d = 0; d < 3; ++d) {
    std::vector<float> x;
    H_TRY(down(a[d], C, x));
    for (int c = 0; c < C; ++c) {
      va[(size_t)d * C + c] = x[c];
      vi[(size_t)d * C + c] = 1.0f / (x[c] + 1e-9f);
    }
  }
  H_TRY(up(h, va, al));
  return up(h, vi, inv);
}

int create_impl(t2w_hift* h, const float* const* W) {
  const t2w_hift_config& c = h->cfg;
  const float* const* w = W;
  int i = 0;
  auto next = [&]() { return w[i++]; };
  h->f0_layers = c.f0_layers;
  for (int l = 0; l < c.f0_layers; ++l) {
    const float* wt = next();
    const float* bt = next();
    H_TRY(conv(h, wt, bt, c.f0_channels, l == 0 ? c.mel : c.f0_channels, 3, &h->f0c[l]));
  }
  {
    const float* wt = next();
    const float* bt = next();
    H_TRY(conv(h, wt, bt, 1, c.f0_channels, 1, &h->f0head));
  }
  {
    std::vector<float> lw, lb;
    H_TRY(down(next(), c.harmonics + 1, lw));
    H_TRY(down(next(), 1, lb));
    H_TRY(up(h, lw, &h->lin_w));
    h->lin_b = lb[0];
  }
  {
    const float* wt = next();
    const float* bt = next();
    H_TRY(conv(h, wt, bt, c.channels, c.mel, 7, &h->pre));
  }
  const int rates[3] = {c.up_rates[0], c.up_rates[1], c.up_rates[2]};
  int cum = 1;
  for (int s = 1; s < 3; ++s) cum *= rates[s];  // 15 for 8, 5, 3
  for (int s = 0; s < 3; ++s) {
    HStage& g = h->st[s];
    g.u = rates[s];
    g.k = c.up_kernels[s];
    g.pad = (g.k - g.u) / 2;
    g.Cin = c.channels >> s;
    g.Cout = c.channels >> (s + 1);
    // ConvTranspose1d weight [Cin, Cout, k]: output t = u m - pad + j reads input m; phase p = t mod u uses taps
    // j = (p + pad) mod u + u q, input index m = (t + pad - j) / u = v + c_p - q for t = u v + p
    std::vector<float> hw, hb;
    H_TRY(down(next(), (size_t)g.Cin * g.Cout * g.k, hw));
    H_TRY(down(next(), g.Cout, hb));
    H_TRY(up(h, hb, &g.b));
    g.phase.resize(g.u);
    g.nq.resize(g.u);
    g.c.resize(g.u);
    for (int p = 0; p < g.u; ++p) {
      const int j0 = (p + g.pad) % g.u;
      const int nq = (g.k - j0 + g.u - 1) / g.u;
      g.nq[p] = nq;
      g.c[p] = (p + g.pad - j0) / g.u;
      // taps in ascending input offset: tap t reads input v + c_p - (nq - 1) + t, i.e. q = nq - 1 - t
      std::vector<float> t((size_t)g.Cout * nq * g.Cin);
      for (int o = 0; o < g.Cout; ++o)
        for (int tt = 0; tt < nq; ++tt)
          for (int ci = 0; ci < g.Cin; ++ci)
            t[((size_t)o * nq + tt) * g.Cin + ci] = hw[((size_t)ci * g.Cout + o) * g.k + j0 + g.u * (nq - 1 - tt)];
      g.phase[p].Cin = g.Cin;
      g.phase[p].Cout = g.Cout;
      g.phase[p].k = nq;
      H_TRY(up(h, t, &g.phase[p].W));
      g.phase[p].b = g.b;
    }
  }
  // source_downs and source ResBlocks
  for (int s = 0; s < 3; ++s) {
    HStage& g = h->st[s];
    const int u = s == 0 ? cum : (s == 1 ? rates[2] : 1);
    const int k = u == 1 ? 1 : 2 * u;
    g.down_stride = u;
    g.down_pad = u == 1 ? 0 : u / 2;
    const float* wt = next();
    const float* bt = next();
    H_TRY(conv(h, wt, bt, g.Cout, kNfft + 2, k, &g.down));
    if (h->tf32) H_TRY(grouped_down(h, g, s));
    HRes& r = g.src;
    r.k = c.source_kernels[s];
    const float* a1[3];
    const float* a2[3];
    for (int d = 0; d < 3; ++d) {
      const float* w1 = next();
      const float* b1 = next();
      H_TRY(conv(h, w1, b1, g.Cout, g.Cout, r.k, &r.c1[d]));
    }
    for (int d = 0; d < 3; ++d) {
      const float* w2 = next();
      const float* b2 = next();
      H_TRY(conv(h, w2, b2, g.Cout, g.Cout, r.k, &r.c2[d]));
    }
    for (int d = 0; d < 3; ++d) a1[d] = next();
    for (int d = 0; d < 3; ++d) a2[d] = next();
    H_TRY(snake_params(h, a1, g.Cout, &r.a1, &r.i1));
    H_TRY(snake_params(h, a2, g.Cout, &r.a2, &r.i2));
  }
  for (int s = 0; s < 3; ++s)
    for (int j = 0; j < 3; ++j) {
      HStage& g = h->st[s];
      HRes& r = g.res[j];
      r.k = c.res_kernels[j];
      const float* a1[3];
      const float* a2[3];
      for (int d = 0; d < 3; ++d) {
        const float* w1 = next();
        const float* b1 = next();
        H_TRY(conv(h, w1, b1, g.Cout, g.Cout, r.k, &r.c1[d]));
      }
      for (int d = 0; d < 3; ++d) {
        const float* w2 = next();
        const float* b2 = next();
        H_TRY(conv(h, w2, b2, g.Cout, g.Cout, r.k, &r.c2[d]));
      }
      for (int d = 0; d < 3; ++d) a1[d] = next();
      for (int d = 0; d < 3; ++d) a2[d] = next();
      H_TRY(snake_params(h, a1, g.Cout, &r.a1, &r.i1));
      H_TRY(snake_params(h, a2, g.Cout, &r.a2, &r.i2));
    }
  {
    const float* wt = next();
    const float* bt = next();
    H_TRY(conv(h, wt, bt, kNfft + 2, c.channels >> 3, 7, &h->post));
  }
  // the fp32 layers outside the upsampling stages on the tensor cores in split form, where their shapes allow
  if (h->tf32) {
    const int fc = c.f0_channels;
    h->f0_tc = c.f0_layers > 1 && (fc % 128 == 0 || fc == 64 || fc == 32);
    for (int l = 1; l < c.f0_layers && h->f0_tc; ++l) H_TRY(split_weights(h, h->f0c[l], fc, &h->f0s[l], nullptr));
    h->post_tc = (c.channels >> 3) % 32 == 0 && kNfft + 2 <= 32;
    if (h->post_tc) H_TRY(split_weights(h, h->post, 32, &h->post_ws, &h->post_bs));
    if ((3 * c.mel) % 4 == 0) {  // conv_pre and f0 layer 1 over the tripled mel rows
      H_TRY(x3_weights(h, h->pre, &h->pre_x3));
      H_TRY(x3_weights(h, h->f0c[0], &h->f00_x3));
    }
  }
  if (h->x3) {  // every stage convolution in split form
    for (int s = 0; s < 3; ++s) {
      HStage& g = h->st[s];
      for (auto& ph : g.phase) H_TRY(split_weights(h, ph, ph.Cout, &ph.Ws, nullptr));
      H_TRY(grouped_down(h, g, s, true));
      HRes* rs[4] = {&g.src, &g.res[0], &g.res[1], &g.res[2]};
      for (HRes* r : rs)
        for (int d = 0; d < 3; ++d) {
          H_TRY(split_weights(h, r->c1[d], r->c1[d].Cout, &r->c1[d].Ws, nullptr));
          H_TRY(split_weights(h, r->c2[d], r->c2[d].Cout, &r->c2[d].Ws, nullptr));
        }
    }
  }
  // window (periodic Hann), cos / sin tables of 2 pi k / 16, Hamming cross-fade window (float64, as np.hamming)
  std::vector<float> tw(48);
  for (int k = 0; k < 16; ++k) {
    tw[k] = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * k / 16.0));
    tw[16 + k] = (float)std::cos(2.0 * M_PI * k / 16.0);
    tw[32 + k] = (float)std::sin(2.0 * M_PI * k / 16.0);
  }
  H_TRY(up(h, tw, &h->tw));
  std::vector<double> hm(2 * kSrcCache);
  for (int n = 0; n < 2 * kSrcCache; ++n) hm[n] = 0.54 - 0.46 * std::cos(2.0 * M_PI * n / (2 * kSrcCache - 1));
  H_TRY(halloc(h, &h->hamming, hm.size()));
  H_CUDA(cudaMemcpy(h->hamming, hm.data(), hm.size() * 8, cudaMemcpyHostToDevice));
  H_TRY(halloc(h, &h->err, 1));
  H_CUDA(cudaMemset(h->err, 0, 4));
  {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = h->device;
    H_CUDA(cudaMemPoolCreate(&h->pool, &props));
    uint64_t keep = UINT64_MAX;
    H_CUDA(cudaMemPoolSetAttribute(h->pool, cudaMemPoolAttrReleaseThreshold, &keep));
  }
  h->cache_ld = kMelCache * c.mel + 2 * kSrcCache;
  H_TRY(halloc(h, &h->cache, (size_t)h->n_streams * h->cache_ld));
  H_CUDA(cudaMemset(h->cache, 0, (size_t)h->n_streams * h->cache_ld * 4));
  for (int r = h->n_streams - 1; r >= 0; --r) h->row_free.push_back(r);
  h->row_live.assign(h->n_streams, 0);
  h->row_first.assign(h->n_streams, 1);
  return T2W_OK;
}

void free_all(t2w_hift* h) {
  for (void* p : h->allocs) cudaFree(p);
  h->allocs.clear();
  for (auto& sg : h->staging) {
    if (sg.host) cudaFreeHost(sg.host);
    if (sg.done) cudaEventDestroy(sg.done);
    sg = t2w_hift::Staging();
  }
  if (h->pool) cudaMemPoolDestroy(h->pool);
  h->pool = nullptr;
  for (auto& kv : h->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.ws) cudaFree(kv.second.ws);
    if (kv.second.done) cudaEventDestroy(kv.second.done);
  }
  h->graphs.clear();
  if (h->cap_stream) cudaStreamDestroy(h->cap_stream);
  h->cap_stream = nullptr;
  if (h->side) cudaStreamDestroy(h->side);
  if (h->fork_ev) cudaEventDestroy(h->fork_ev);
  if (h->join_ev) cudaEventDestroy(h->join_ev);
  h->side = nullptr;
  h->fork_ev = h->join_ev = nullptr;
  for (int k = 0; k < 2; ++k) {
    if (h->res_st[k]) cudaStreamDestroy(h->res_st[k]);
    if (h->res_ev[k]) cudaEventDestroy(h->res_ev[k]);
    h->res_st[k] = nullptr;
    h->res_ev[k] = nullptr;
  }
}

// ---- a call's plan
struct HPlan {
  int n = 0;
  std::vector<HRow> rows;
  int R[4] = {};  // rows at the mel rate and the three stage rates
  int A[4] = {};  // allocated rows: the mel rate rounded up to 128, the stages its 8, 40 and 120 multiples
  std::vector<int> vs_mel, vs_s[3];  // virtual rows (the windows' data rows back to back) per rate: prefix offsets
  std::vector<int> start_mel, len_mel, start_s[3], len_s[3], start_up[3];
  long long samples = 0, out_samples = 0;
};

int make_plan(t2w_hift* h, int n, const int32_t* handle, const int32_t* T, const uint8_t* last, HPlan& pl) {
  pl = HPlan();
  pl.n = n;
  pl.vs_mel.assign(1, 0);
  for (int s = 0; s < 3; ++s) pl.vs_s[s].assign(1, 0);
  const int up = (int)(h->cfg.up_rates[0] * h->cfg.up_rates[1] * h->cfg.up_rates[2]) * kHop;  // 480
  int rm = 0, r0 = 0, r1 = 0, r2 = 0, mel_off = 0;
  long long smp = 0, outp = 0;
  for (int i = 0; i < n; ++i) {
    const int row = handle[i];
    const bool first = h->row_first[row] != 0;
    const int F = T[i] + (first ? 0 : kMelCache);
    if (T[i] <= 0 || F > h->max_frames || (!last[i] && F < kMelCache)) return T2W_ERR_INVALID;
    const int N = F * up;
    HRow e{};
    e.F = F;
    e.first = first;
    e.cache = row;
    e.mel_off = mel_off;
    e.mel0 = rm + kPadMel;
    e.s0 = r0 + 8 * kPadMel;
    e.s1 = r1 + 40 * kPadMel;
    e.s2 = r2 + 120 * kPadMel - 1;
    e.smp0 = (int)smp;
    e.last = last[i] != 0;
    e.out0 = (int)outp;
    e.out_len = e.last ? N : (first ? N : N - kSrcCache);
    pl.rows.push_back(e);
    pl.vs_mel.push_back(pl.vs_mel.back() + F);
    pl.vs_s[0].push_back(pl.vs_s[0].back() + 8 * F);
    pl.vs_s[1].push_back(pl.vs_s[1].back() + 40 * F);
    pl.vs_s[2].push_back(pl.vs_s[2].back() + 120 * F + 1);
    pl.start_mel.push_back(e.mel0);
    pl.len_mel.push_back(F);
    pl.start_s[0].push_back(e.s0);
    pl.len_s[0].push_back(8 * F);
    pl.start_s[1].push_back(e.s1);
    pl.len_s[1].push_back(40 * F);
    pl.start_s[2].push_back(e.s2);
    pl.len_s[2].push_back(120 * F + 1);
    // the transposed conv of stage s writes output row u v + p at the stage's data start (stage 2: after the
    // reflection row)
    pl.start_up[0].push_back(e.s0);
    pl.start_up[1].push_back(e.s1);
    pl.start_up[2].push_back(e.s2 + 1);
    rm += F + 2 * kPadMel;
    r0 += 8 * (F + 2 * kPadMel);
    r1 += 40 * (F + 2 * kPadMel);
    r2 += 120 * (F + 2 * kPadMel);
    mel_off += T[i];
    smp += N;
    outp += e.out_len;
  }
  pl.R[0] = rm;
  pl.R[1] = r0;
  pl.R[2] = r1;
  pl.R[3] = r2;
  pl.A[0] = (rm + 127) / 128 * 128;
  pl.A[1] = 8 * pl.A[0];
  pl.A[2] = 40 * pl.A[0];
  pl.A[3] = 120 * pl.A[0];
  pl.samples = smp;
  pl.out_samples = outp;
  return T2W_OK;
}

// The per-row padding flags of each rate (1 unless the row holds a window's data), written into dst[r] (A[r] bytes).
void fill_pads(const HPlan& pl, uint8_t* const dst[4]) {
  for (int r = 0; r < 4; ++r) std::memset(dst[r], 1, pl.A[r]);
  for (const HRow& e : pl.rows) {
    std::memset(dst[0] + e.mel0, 0, e.F);
    std::memset(dst[1] + e.s0, 0, 8 * e.F);
    std::memset(dst[2] + e.s1, 0, 40 * e.F);
    std::memset(dst[3] + e.s2, 0, 120 * e.F + 1);
  }
}

}  // namespace

extern "C" {

int t2w_hift_create(const t2w_hift_config* cfg, const float* const* weights, int32_t n_weights, int32_t max_frames,
                    int32_t n_streams, t2w_hift** out) {
  // window rows are tagged (stream << 20 | row) in 32-bit words: at most 2047 streams
  if (!cfg || !weights || !out || n_streams <= 0 || n_streams > 2047 || max_frames < kMelCache + 1 || max_frames > 4096)
    return T2W_ERR_INVALID;
  const t2w_hift_config& c = *cfg;
  if (c.tf32 < 0 || c.tf32 > 2) return T2W_ERR_INVALID;
  if (c.mel <= 0 || c.channels % 64 || c.channels < 64 || c.f0_layers < 1 || c.f0_layers > 8 || c.harmonics + 1 > kMaxHarm ||
      c.n_fft != kNfft || c.hop != kHop || c.up_rates[0] * c.up_rates[1] * c.up_rates[2] * kHop != 480 ||
      c.up_rates[0] != 8 || c.up_rates[1] != 5 || c.up_rates[2] != 3)
    return T2W_ERR_UNSUPPORTED;
  for (int s = 0; s < 3; ++s)
    if (c.up_kernels[s] - c.up_rates[s] < 0 || (c.up_kernels[s] - c.up_rates[s]) % 2 ||
        c.up_kernels[s] - 2 * ((c.up_kernels[s] - c.up_rates[s]) / 2) != c.up_rates[s])
      return T2W_ERR_UNSUPPORTED;
  if (max_frames > kMaxFrames) return T2W_ERR_INVALID;
  const int expect = 2 * c.f0_layers + 2 + 2 + 2 + 3 * 2 + 3 * (2 + 18) + 9 * 18 + 2;
  if (n_weights != expect) return T2W_ERR_INVALID;
  for (int i = 0; i < n_weights; ++i)
    if (!weights[i]) return T2W_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || !t2w_device_ok(dev)) return T2W_ERR_UNSUPPORTED;
  t2w_hift* h = new t2w_hift();
  h->cfg = c;
  h->device = dev;
  h->n_streams = n_streams;
  h->max_frames = max_frames;
  h->x3 = c.tf32 == 2;
  h->tc_parts = h->x3 ? 0x1FFu : c.tf32 ? (c.tf32_parts ? (c.tf32_parts & 0x1FFu) : 0x1FFu) : 0u;
  h->tf32 = h->tc_parts != 0;
  const int rc = create_impl(h, weights);
  if (rc) {
    free_all(h);
    delete h;
    return rc;
  }
  *out = h;
  return T2W_OK;
}

int t2w_hift_destroy(t2w_hift* h) {
  if (!h) return T2W_ERR_INVALID;
  cudaDeviceSynchronize();
  free_all(h);
  delete h;
  return T2W_OK;
}

int t2w_hift_check(t2w_hift* h) {
  if (!h) return T2W_ERR_INVALID;
  int v = 0;
  H_CUDA(cudaMemcpy(&v, h->err, 4, cudaMemcpyDeviceToHost));
  if (v) {
    const int z = 0;
    H_CUDA(cudaMemcpy(h->err, &z, 4, cudaMemcpyHostToDevice));
  }
  return v;
}

int t2w_hift_stream_new(t2w_hift* h, int32_t* handle) {
  if (!h || !handle) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lk(h->mu);
  if (h->row_free.empty()) return T2W_ERR_EXHAUSTED;
  const int r = h->row_free.back();
  h->row_free.pop_back();
  h->row_live[r] = 1;
  h->row_first[r] = 1;
  *handle = r;
  return T2W_OK;
}

int t2w_hift_stream_release(t2w_hift* h, int32_t handle) {
  if (!h || handle < 0 || handle >= h->n_streams) return T2W_ERR_INVALID;
  std::lock_guard<std::mutex> lk(h->mu);
  if (!h->row_live[handle]) return T2W_ERR_INVALID;
  h->row_live[handle] = 0;
  h->row_free.push_back(handle);
  return T2W_OK;
}

int64_t t2w_vocode_samples(const t2w_hift* h, int32_t n, const int32_t* handle, const int32_t* T, const uint8_t* last,
                           int64_t* per_stream, int32_t* frames) {
  if (!h || n <= 0 || !handle || !T || !last) return -1;
  std::lock_guard<std::mutex> lk(const_cast<t2w_hift*>(h)->mu);
  long long tot = 0;
  for (int i = 0; i < n; ++i) {
    if (handle[i] < 0 || handle[i] >= h->n_streams || !h->row_live[handle[i]] || T[i] <= 0) return -1;
    const bool first = h->row_first[handle[i]] != 0;
    const long long N = 480ll * (T[i] + (first ? 0 : kMelCache));
    const long long o = last[i] ? N : (first ? N : N - kSrcCache);
    if (per_stream) per_stream[i] = o;
    if (frames) frames[i] = T[i] + (first ? 0 : kMelCache);
    tot += o;
  }
  return tot;
}

int t2w_vocode(t2w_hift* h, const t2w_vocode_batch* b, void* stream) {
  if (!h || !b || b->n_streams <= 0 || !b->handle || !b->T || !b->last || !b->mel || !b->rand_ini || !b->noise || !b->out)
    return T2W_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lk(h->mu);
  const int n = b->n_streams;
  for (int i = 0; i < n; ++i) {
    if (b->handle[i] < 0 || b->handle[i] >= h->n_streams || !h->row_live[b->handle[i]]) return T2W_ERR_INVALID;
    for (int j = 0; j < i; ++j)
      if (b->handle[j] == b->handle[i]) return T2W_ERR_INVALID;
  }
  if (!h->side) {  // once: the streams of the call's independent branches, and their fork / join events
    cudaError_t e = cudaStreamCreateWithFlags(&h->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->fork_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->join_ev, cudaEventDisableTiming);
    for (int k = 0; k < 2; ++k) {
      if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->res_st[k], cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->res_ev[k], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
      set_cuda_error(e);
      if (h->side) cudaStreamDestroy(h->side);
      if (h->fork_ev) cudaEventDestroy(h->fork_ev);
      if (h->join_ev) cudaEventDestroy(h->join_ev);
      h->side = nullptr;
      h->fork_ev = h->join_ev = nullptr;
      for (int k = 0; k < 2; ++k) {
        if (h->res_st[k]) cudaStreamDestroy(h->res_st[k]);
        if (h->res_ev[k]) cudaEventDestroy(h->res_ev[k]);
        h->res_st[k] = nullptr;
        h->res_ev[k] = nullptr;
      }
      return T2W_ERR_CUDA;
    }
  }
  HPlan pl;
  H_TRY(make_plan(h, n, b->handle, b->T, b->last, pl));
  const t2w_hift_config& c = h->cfg;
  const int C0 = c.channels;
  // device buffers for this call (stream-ordered allocations)
  size_t meta = 0;
  auto add = [&](size_t bytes) {
    const size_t o = meta;
    meta = a256(meta + bytes);
    return o;
  };
  const size_t o_rows = add(pl.rows.size() * sizeof(HRow));
  const size_t o_vm = add((n + 1) * 4), o_sm = add(n * 4), o_lm = add(n * 4);
  size_t o_vs[3], o_ss[3], o_ls[3], o_su[3];
  for (int s = 0; s < 3; ++s) {
    o_vs[s] = add((n + 1) * 4);
    o_ss[s] = add(n * 4);
    o_ls[s] = add(n * 4);
    o_su[s] = add(n * 4);
  }
  size_t o_pad[4];
  for (int r = 0; r < 4; ++r) o_pad[r] = add(pl.A[r]);
  const size_t meta_bytes = meta;
  const size_t o_mel = add((size_t)pl.A[0] * c.mel * 4);
  // the f0 layers' activations, [hi | lo] pairs (2 x f0_channels floats per row) when they feed the split-form convs
  const size_t o_f0a = add((size_t)pl.A[0] * c.f0_channels * 8), o_f0b = add((size_t)pl.A[0] * c.f0_channels * 8);
  const size_t o_f0 = add((size_t)pl.A[0] * 4);
  const size_t o_src = add((size_t)pl.samples * 4), o_sp = add((size_t)pl.samples * 4);
  const int fc = c.f0_channels;
  auto tc_n = [](int N) { return N % 128 == 0 || N == 64 || N == 32; };  // widths the tensor-core conv takes
  const bool pre_tc = h->pre_x3 && tc_n(C0), f00_tc = h->f00_x3 && tc_n(fc);
  const size_t o_mel3 = (pre_tc || f00_tc) ? add((size_t)pl.A[0] * 3 * c.mel * 4) : 0;
  const int stft_ld = h->x3 ? kStftLd3 : kStftLd;
  const size_t o_stft = add((size_t)pl.A[3] * stft_ld * 4);
  const int xsm = h->x3 ? 2 : 1;  // the fp32 tensor-core mode keeps conv inputs as [hi | lo] pairs: twice the floats
  const size_t o_x0 = add((size_t)pl.A[0] * C0 * 4 * xsm);
  // per stage: x (ups output), xr[3] ResBlock streams, ar[3] / sd scratch of the stage's size
  // (tx[2]: the scratch of ResBlocks 1 and 2, which run beside ResBlock 0 and its scratch ta)
  size_t o_xs[3], o_xr[3][3], o_ar[3][3], o_sd[3], o_ta[3], o_tx[3][2];
  for (int s = 0; s < 3; ++s) {
    const size_t sz = (size_t)pl.A[s + 1] * (C0 >> (s + 1)) * 4;
    o_xs[s] = add(sz);
    for (int j = 0; j < 3; ++j) o_xr[s][j] = add(sz);
    for (int j = 0; j < 3; ++j) o_ar[s][j] = add(sz * xsm);
    o_sd[s] = add(sz * xsm);
    o_ta[s] = add(sz * xsm);
    for (int k = 0; k < 2; ++k) o_tx[s][k] = add(sz * xsm);
  }
  const int post_ld = h->post_tc ? 32 : kNfft + 2;  // conv_post's output (18 columns; 32 on the tensor cores)
  const size_t o_post = add((size_t)pl.A[3] * post_ld * 4);
  // stage 2's output as [hi | lo] pairs, conv_post's input in split form
  const size_t o_xps = h->post_tc ? add((size_t)pl.A[3] * (C0 >> 3) * 8) : 0;
  // a graph call reads the window's mel and noise from, and writes its samples to, buffers of its own workspace
  const bool graph = (b->flags & T2W_FLAG_GRAPH) != 0;
  long long mel_rows = 0;
  for (int i = 0; i < n; ++i) mel_rows += b->T[i];
  const int dim = c.harmonics + 1;
  const size_t o_gmel = graph ? add((size_t)mel_rows * c.mel * 4) : 0;
  const size_t o_gnoise = graph ? add((size_t)pl.samples * dim * 4) : 0;
  const size_t o_gout = graph ? add((size_t)pl.out_samples * 4) : 0;
  const size_t total = meta;
  // the launches depend only on the call's sizes (every window's rows, handles and padding flags are data in the
  // workspace): one graph per size key, captured the second time the key is seen
  t2w_hift::Graph* hg = nullptr;
  bool capture = false;
  uint64_t key = 0;
  if (graph) {
    key = 0x41F7ull;
    for (long long v : {(long long)n, (long long)pl.A[0], (long long)pl.vs_mel[n], (long long)pl.vs_s[0][n],
                        (long long)pl.vs_s[1][n], (long long)pl.vs_s[2][n], pl.samples, pl.out_samples, mel_rows})
      key = (key ^ ((uint64_t)v + 0x9e3779b97f4a7c15ull + (key << 6) + (key >> 2))) * 0xff51afd7ed558ccdull;
    auto it = h->graphs.find(key);
    if (it != h->graphs.end()) {
      hg = &it->second;
    } else {
      cudaStreamCaptureStatus cs;
      H_CUDA(cudaStreamIsCapturing(st, &cs));
      if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;  // the caller is capturing: flags = 0
      if (h->seen.size() > 4096) h->seen.clear();
      if (++h->seen[key] >= 2) {
        if (h->graphs.size() >= 16) {  // drop one, once its latest launch has finished
          auto victim = h->graphs.begin();
          H_CUDA(cudaEventSynchronize(victim->second.done));
          cudaGraphExecDestroy(victim->second.exec);
          cudaFree(victim->second.ws);
          cudaEventDestroy(victim->second.done);
          h->graphs.erase(victim);
        }
        t2w_hift::Graph ng;
        H_CUDA(cudaMalloc(reinterpret_cast<void**>(&ng.ws), total));
        const cudaError_t ee = cudaEventCreateWithFlags(&ng.done, cudaEventDisableTiming);
        if (ee != cudaSuccess) {
          cudaFree(ng.ws);
          set_cuda_error(ee);
          return T2W_ERR_CUDA;
        }
        hg = &h->graphs.emplace(key, ng).first->second;
        capture = true;
      }
    }
  }
  uint8_t* ws = nullptr;
  if (hg)
    ws = hg->ws;
  else
    H_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), total, h->pool, st));
  auto P = [&](size_t o) { return ws + o; };
  auto drop_graph = [&]() {  // a capture that failed leaves no entry behind
    if (capture) {
      if (hg->exec) cudaGraphExecDestroy(hg->exec);
      cudaFree(hg->ws);
      cudaEventDestroy(hg->done);
      h->graphs.erase(key);
      hg = nullptr;
    }
  };
  // the plan's image in a pinned staging buffer, rewritten only after the copy that last read it has completed
  t2w_hift::Staging& sg = h->staging[h->staging_next];
  h->staging_next = (h->staging_next + 1) % t2w_hift::kStaging;
  cudaError_t se = cudaSuccess;
  if (sg.used) se = cudaEventSynchronize(sg.done);
  if (se == cudaSuccess && sg.cap < meta_bytes) {
    if (sg.host) cudaFreeHost(sg.host);
    sg.host = nullptr;
    sg.cap = 0;
    const size_t cap = std::max<size_t>(2 * meta_bytes, 1 << 16);  // room for longer windows before it grows again
    se = cudaMallocHost(&sg.host, cap);
    if (se == cudaSuccess) sg.cap = cap;
  }
  if (se == cudaSuccess && !sg.done) se = cudaEventCreateWithFlags(&sg.done, cudaEventDisableTiming);
  if (se != cudaSuccess) {
    set_cuda_error(se);
    if (hg)
      drop_graph();
    else
      cudaFreeAsync(ws, st);
    return T2W_ERR_CUDA;
  }
  uint8_t* img = static_cast<uint8_t*>(sg.host);
  auto put = [&](size_t o, const void* s, size_t bytes) {
    if (bytes) std::memcpy(img + o, s, bytes);
  };
  put(o_rows, pl.rows.data(), pl.rows.size() * sizeof(HRow));
  put(o_vm, pl.vs_mel.data(), (n + 1) * 4);
  put(o_sm, pl.start_mel.data(), n * 4);
  put(o_lm, pl.len_mel.data(), n * 4);
  for (int s = 0; s < 3; ++s) {
    put(o_vs[s], pl.vs_s[s].data(), (n + 1) * 4);
    put(o_ss[s], pl.start_s[s].data(), n * 4);
    put(o_ls[s], pl.len_s[s].data(), n * 4);
    put(o_su[s], pl.start_up[s].data(), n * 4);
  }
  {
    uint8_t* const pads[4] = {img + o_pad[0], img + o_pad[1], img + o_pad[2], img + o_pad[3]};
    fill_pads(pl, pads);
  }
  {
    cudaError_t e0 = cudaMemcpyAsync(ws, img, meta_bytes, cudaMemcpyHostToDevice, st);
    if (e0 == cudaSuccess) e0 = cudaEventRecord(sg.done, st);
    if (e0 == cudaSuccess) sg.used = true;
    if (graph && e0 == cudaSuccess)
      e0 = cudaMemcpyAsync(ws + o_gmel, b->mel, (size_t)mel_rows * c.mel * 4, cudaMemcpyDeviceToDevice, st);
    if (graph && e0 == cudaSuccess && b->noise_ready)  // the caller's noise draws, before the copy reads them
      e0 = cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(b->noise_ready), 0);
    if (graph && e0 == cudaSuccess)
      e0 = cudaMemcpyAsync(ws + o_gnoise, b->noise, (size_t)pl.samples * dim * 4, cudaMemcpyDeviceToDevice, st);
    if (e0 != cudaSuccess) {
      set_cuda_error(e0);
      if (hg)
        drop_graph();
      else
        cudaFreeAsync(ws, st);
      return T2W_ERR_CUDA;
    }
  }
  const float* in_mel = graph ? reinterpret_cast<const float*>(ws + o_gmel) : b->mel;
  const float* in_noise = graph ? reinterpret_cast<const float*>(ws + o_gnoise) : b->noise;
  float* out_samples = graph ? reinterpret_cast<float*>(ws + o_gout) : b->out;
  const HRow* drows = reinterpret_cast<const HRow*>(P(o_rows));
  float* mel = reinterpret_cast<float*>(P(o_mel));
  float* src = reinterpret_cast<float*>(P(o_src));
  float* speech = reinterpret_cast<float*>(P(o_sp));
  // every launch of the call, on `st` (the caller's stream, or the capture stream of a graph)
  auto enqueue = [&](cudaStream_t st) -> int {
  int rc = T2W_OK;
  const cudaStream_t st_main = st;
  bool forked = false;      // the second stream has work the caller's stream has not waited for
  bool res_forked = false;  // so have the ResBlock streams
  auto fail = [&](int r) {
    if (forked) {  // join before returning: the caller frees or drops the workspace on its own stream
      cudaEventRecord(h->join_ev, h->side);
      cudaStreamWaitEvent(st_main, h->join_ev, 0);
      forked = false;
    }
    if (res_forked) {
      for (int k = 0; k < 2; ++k) {
        cudaEventRecord(h->res_ev[k], h->res_st[k]);
        cudaStreamWaitEvent(st_main, h->res_ev[k], 0);
      }
      res_forked = false;
    }
    return r;
  };
  {
    cudaError_t e1 = cudaSuccess;
    // buffers whose rows around the windows' data must read as zero and that no kernel writes in full: the mel rows and
    // conv_pre's output (read by the transposed conv's tensor-map loads), the source branch and its Snake (added to
    // every row by the fan-out; read by the ResBlock convs), and the transposed conv's output when the fp32 kernel,
    // which writes data rows only, makes it; and the first f0 layer's output when the split-form convs read it
    auto zero = [&](size_t off, size_t bytes) {
      if (e1 == cudaSuccess) e1 = cudaMemsetAsync(ws + off, 0, bytes, st);
    };
    zero(o_mel, (size_t)pl.A[0] * c.mel * 4);
    if (h->f0_tc) zero(o_f0a, (size_t)pl.A[0] * c.f0_channels * 8);
    zero(o_x0, (size_t)pl.A[0] * C0 * 4);
    // (the parts on CUDA cores write data rows only; with some part on the tensor cores, whose tensor maps read
    // padding rows, the ResBlock streams of a CUDA-core ResBlock part too, as the average of them feeds the next stage)
    if (h->tc_parts & 0x92u)
      zero(o_stft, (size_t)pl.A[3] * stft_ld * 4);  // the source_down tensor maps read padding rows and channels
    if (o_mel3) zero(o_mel3, (size_t)pl.A[0] * 3 * c.mel * 4);
    for (int s = 0; s < 3; ++s) {
      const size_t sz = (size_t)pl.A[s + 1] * (C0 >> (s + 1)) * 4;
      if (!(h->tc_parts >> (3 * s + 1) & 1u)) {
        zero(o_sd[s], sz);
        zero(o_ta[s], sz);
        for (int k = 0; k < 2; ++k) zero(o_tx[s][k], sz);
      }
      if (!(h->tc_parts >> (3 * s) & 1u)) zero(o_xs[s], sz);
      if (h->tf32 && !(h->tc_parts >> (3 * s + 2) & 1u))
        for (int j = 0; j < 3; ++j) zero(o_xr[s][j], sz);
    }
    if (e1 != cudaSuccess) {
      set_cuda_error(e1);
      return fail(T2W_ERR_CUDA);
    }
  }
  auto run = [&](ConvGeo g) -> int {
    if (g.nv <= 0) return T2W_OK;
    if (g.Cout <= 32) {
      dim3 grid((g.nv + 127) / 128, (g.Cout + 31) / 32);
      return ck(launch_k(k_hconv<128, 32>, grid, dim3(256), 0, st, g));
    }
    dim3 grid((g.nv + 63) / 64, (g.Cout + 63) / 64);
    return ck(launch_k(k_hconv<64, 64>, grid, dim3(256), 0, st, g));
  };
  auto geo = [&](const HConv& cv, const int* vr, int nv, const int* in_s, const int* in_l, const int* out_s,
                 const float* in, float* outp, int epi) {
    ConvGeo g;
    g.vstart = vr;
    g.nstreams = n;
    g.nv = nv;
    g.in_start = in_s;
    g.in_len = in_l;
    g.out_start = out_s;
    g.in = in;
    g.ld_in = cv.Cin;
    g.Cin = cv.Cin;
    g.out = outp;
    g.ld_out = cv.Cout;
    g.Cout = cv.Cout;
    g.W = cv.W;
    g.bias = cv.b;
    g.taps = cv.k;
    g.stride = 1;
    g.off = -(cv.k / 2);
    g.dil = 1;
    g.epi = epi;
    return g;
  };
  const int* vm = reinterpret_cast<const int*>(P(o_vm));
  const int* sm = reinterpret_cast<const int*>(P(o_sm));
  const int* lm = reinterpret_cast<const int*>(P(o_lm));
  // 1. mel rows
  {
    dim3 grid(h->max_frames, n);
    rc = ck(launch_k(k_mel_in, grid, dim3(128), 0, st, in_mel, drows, (const float*)h->cache, h->cache_ld, c.mel, mel,
                     o_mel3 ? reinterpret_cast<float*>(P(o_mel3)) : nullptr));
    if (rc) return fail(rc);
  }
  // 2 - 4 and every stage's source branch run on the vocoder's second stream, beside conv_pre and the stages'
  // transposed convs and ResBlocks, which share no buffer with them (every buffer of the workspace has its own range;
  // a stage's source-branch buffers are read or reused only from its fan-out on); each fan-out waits for its stage's
  // source branch.  (Graph capture follows the fork and the joins.)
  rc = ck(cudaEventRecord(h->fork_ev, st_main));
  if (rc) return fail(rc);
  rc = ck(cudaStreamWaitEvent(h->side, h->fork_ev, 0));
  if (rc) return fail(rc);
  forked = true;
  st = h->side;
  // 2. f0 predictor: convs + ELU, then |linear|.  On the tensor cores (fp32-level accuracy): the first layer over the
  // tripled mel rows (80 channels), the others in split form; the first writes its ELU output as [hi | lo] pairs, the
  // middle layers read and write pairs, the last writes plain fp32 for the head.
  const uint8_t* pad0 = reinterpret_cast<const uint8_t*>(P(o_pad[0]));
  {
    float* a = reinterpret_cast<float*>(P(o_f0a));
    float* bb = reinterpret_cast<float*>(P(o_f0b));
    const float* in = mel;
    for (int l = 0; l < h->f0_layers; ++l) {
      float* o = (l & 1) ? bb : a;
      const bool split_out = h->f0_tc && l + 1 < h->f0_layers;
      if (l == 0 && f00_tc) {
        TConvArgs t;
        t.A = reinterpret_cast<const float*>(P(o_mel3));
        t.lda = 3 * c.mel;
        t.rows_a = pl.A[0];
        t.W = h->f00_x3;
        t.bias = h->f0c[0].b;
        t.M = pl.A[0];
        t.N = fc;
        t.Cin = 3 * c.mel;
        t.taps = 3;
        t.tap_row0 = -1;
        t.out = o;
        t.ldo = split_out ? 2 * fc : fc;
        t.pad = pad0;
        t.epi = TCONV_ELU;
        t.split_out = split_out;
        t.err = h->err;
        rc = launch_tconv(t, st);
      } else if (l == 0 || !h->f0_tc) {
        ConvGeo cg = geo(h->f0c[l], vm, pl.vs_mel[n], sm, lm, sm, in, o, split_out ? HE_ELU_SPLIT : HE_ELU);
        if (split_out) cg.ld_out = 2 * fc;
        rc = run(cg);
      } else {
        TConvArgs t;
        t.A = in;
        t.lda = 2 * fc;
        t.rows_a = pl.A[0];
        t.W = h->f0s[l];
        t.bias = h->f0c[l].b;
        t.M = pl.A[0];
        t.N = fc;
        t.Cin = fc;
        t.taps = 3;
        t.tap_row0 = -1;
        t.out = o;
        t.ldo = split_out ? 2 * fc : fc;
        t.pad = pad0;
        t.epi = TCONV_ELU;
        t.split_in = 1;
        t.split_out = split_out;
        t.err = h->err;
        rc = launch_tconv(t, st);
      }
      if (rc) return fail(rc);
      in = o;
    }
    const int ld = h->f0c[h->f0_layers - 1].Cout;
    rc = ck(launch_k(k_f0_head, dim3((pl.A[0] + 7) / 8), dim3(256), 0, st, in, ld, fc, (const float*)h->f0head.W,
                     (const float*)h->f0head.b, pad0, pl.A[0], reinterpret_cast<float*>(P(o_f0))));
    if (rc) return fail(rc);
  }
  // 3. the harmonic source, 4. its STFT
  float* stft = reinterpret_cast<float*>(P(o_stft));
  {
    const dim3 sgrid((480 * h->max_frames + kSrcChunk - 1) / kSrcChunk, n);
    if (!graph && b->noise_ready) {  // eager: the caller's noise draws (another stream) before the first read of them
      rc = ck(cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(b->noise_ready), 0));
      if (rc) return fail(rc);
    }
    rc = ck(launch_k(k_source, sgrid, dim3(256), 0, st, (const float*)P(o_f0), drows, in_noise, (const float*)h->lin_w,
                     h->lin_b, c.harmonics + 1, (float)c.sample_rate, 480.f, c.nsf_alpha, c.nsf_sigma, c.voiced_threshold,
                     (const float*)h->cache, h->cache_ld, kMelCache * c.mel, src));
    if (rc) return fail(rc);
    dim3 grid((120 * h->max_frames + 1 + 127) / 128, n);
    rc = ck(launch_k(k_stft, grid, dim3(128), 0, st, (const float*)src, drows, (const float*)h->tw, stft, stft_ld, 480.f,
                     h->x3));
    if (rc) return fail(rc);
  }
  st = st_main;  // the second stream goes on with stage 0's source branch
  // 5. conv_pre
  float* x = reinterpret_cast<float*>(P(o_x0));
  if (pre_tc) {  // over the tripled mel rows: fp32-level products on the tensor cores; the fp32 mode writes pairs
    TConvArgs t;
    t.A = reinterpret_cast<const float*>(P(o_mel3));
    t.lda = 3 * c.mel;
    t.rows_a = pl.A[0];
    t.W = h->pre_x3;
    t.bias = h->pre.b;
    t.M = pl.A[0];
    t.N = C0;
    t.Cin = 3 * c.mel;
    t.taps = h->pre.k;
    t.tap_row0 = -(h->pre.k / 2);
    t.out = x;
    t.ldo = (long long)C0 * xsm;
    t.pad = pad0;
    t.epi = TCONV_LEAKY;  // stage 0's leaky_relu fused
    t.slope = c.lrelu_slope;
    t.split_out = h->x3;
    t.err = h->err;
    rc = launch_tconv(t, st);
    if (rc) return fail(rc);
  } else {
    ConvGeo cg = geo(h->pre, vm, pl.vs_mel[n], sm, lm, sm, mel, x, HE_LEAKY);  // stage 0's leaky_relu fused
    cg.slope = c.lrelu_slope;
    rc = run(cg);
    if (rc) return fail(rc);
  }
  // 6. stages
  const int* vin = vm;
  const int* s_in = sm;
  const int* l_in = lm;
  int nvin = pl.vs_mel[n];
  for (int s = 0; s < 3; ++s) {
    HStage& g = h->st[s];
    const int Cs = g.Cout;
    // x already holds leaky_relu(x) (conv_pre's epilogue, or the previous stage's average)
    float* xs = reinterpret_cast<float*>(P(o_xs[s]));
    const int* vs = reinterpret_cast<const int*>(P(o_vs[s]));
    const int* ss = reinterpret_cast<const int*>(P(o_ss[s]));
    const int* ls = reinterpret_cast<const int*>(P(o_ls[s]));
    const int* su = reinterpret_cast<const int*>(P(o_su[s]));
    const bool ups_tc = h->tc_parts >> (3 * s) & 1u, src_tc = h->tc_parts >> (3 * s + 1) & 1u,
               res_tc = h->tc_parts >> (3 * s + 2) & 1u;
    // transposed conv, one launch per output phase over the input's data rows
    for (int p = 0; p < g.u; ++p) {
      if (ups_tc) {
        TConvArgs t;
        t.A = x;
        t.lda = g.Cin * xsm;
        t.rows_a = pl.A[s];
        t.W = h->x3 ? g.phase[p].Ws : g.phase[p].W;
        t.split_in = h->x3;
        t.bias = g.b;
        t.M = pl.A[s];
        t.N = g.Cout;
        t.Cin = g.Cin;
        t.taps = g.nq[p];
        t.tap_row0 = g.c[p] - (g.nq[p] - 1);
        t.out = xs;
        t.ldo = g.Cout;
        t.row_mul = g.u;
        t.row_add = p;
        t.pad = reinterpret_cast<const uint8_t*>(P(o_pad[s + 1]));
        t.err = h->err;
        rc = launch_tconv(t, st);
      } else {
        ConvGeo cg = geo(g.phase[p], vin, nvin, s_in, l_in, su, x, xs, HE_NONE);
        cg.off = g.c[p] - (g.nq[p] - 1);
        cg.dil = 1;
        cg.u_out = g.u;
        cg.p_out = p;
        rc = run(cg);
      }
      if (rc) return fail(rc);
    }
    if (s == 2) {
      rc = ck(launch_k(k_reflect_row, dim3(n), dim3(64), 0, st, xs, drows, Cs));
      if (rc) return fail(rc);
    }
    // source branch (second stream): strided conv of the STFT, then its ResBlock (in place)
    st = h->side;
    forked = true;
    float* sd = reinterpret_cast<float*>(P(o_sd[s]));
    float* ta = reinterpret_cast<float*>(P(o_ta[s]));
    if (src_tc) {  // TF32 (the source branch is part of the reference's decode_tf32 stages)
      const int S = g.down_stride;
      TConvArgs t;
      t.A = stft;  // viewed as rows of S frames
      t.lda = S * stft_ld;
      t.rows_a = pl.A[3] / S;
      t.W = h->x3 ? g.down_x3 : g.down_tc;
      t.bias = g.down.b;
      t.M = pl.A[s + 1];
      t.N = Cs;
      t.Cin = S * stft_ld;
      t.taps = g.down_taps;
      t.tap_row0 = g.down_q0;
      t.out = sd;
      t.ldo = Cs;
      t.pad = reinterpret_cast<const uint8_t*>(P(o_pad[s + 1]));
      t.alpha = g.src.a1;  // the source ResBlock's first Snake of the branch, written beside it
      t.inv = g.src.i1;
      t.out2 = ta;
      t.split_out2 = h->x3;
      t.ldo2 = (long long)Cs * xsm;
      t.err = h->err;
      rc = launch_tconv(t, st);
      if (rc) return fail(rc);
    } else {
      ConvGeo cg = geo(g.down, vs, pl.vs_s[s][n], reinterpret_cast<const int*>(P(o_ss[2])),
                       reinterpret_cast<const int*>(P(o_ls[2])), ss, stft, sd, HE_NONE);
      cg.ld_in = kStftLd;
      cg.stride = g.down_stride;
      cg.off = -g.down_pad;
      cg.alpha = g.src.a1;  // the source ResBlock's first Snake of the branch, written beside it
      cg.inv = g.src.i1;
      cg.out2 = ta;
      rc = run(cg);
      if (rc) return fail(rc);
    }
    const long long nel = (long long)pl.A[s + 1] * Cs;
    auto resblock = [&](HRes& r, float* xr, float* a_in, float* tmp, const float* base, bool tc) -> int {
      // a_in holds Snake1_0(x); per dilation: tmp = Snake2(conv1(a_in)); xr = x + conv2(tmp), a_in = Snake1_next(xr),
      // x = base for the first dilation when given (xr written out of place), else xr itself
      for (int dd = 0; dd < 3; ++dd) {
        const int dl = h->cfg.dilations[dd];
        if (tc) {
          TConvArgs t;
          t.lda = Cs;
          t.rows_a = pl.A[s + 1];
          t.M = pl.A[s + 1];
          t.N = Cs;
          t.Cin = Cs;
          t.taps = r.k;
          t.ldo = Cs;
          t.pad = reinterpret_cast<const uint8_t*>(P(o_pad[s + 1]));
          t.err = h->err;
          // the fp32 tensor-core mode: the Snake outputs (conv inputs) as [hi | lo] pairs, the convs in split form
          t.lda = Cs * xsm;
          t.split_in = h->x3;
          TConvArgs t1 = t;
          t1.A = a_in;
          t1.W = h->x3 ? r.c1[dd].Ws : r.c1[dd].W;
          t1.ldo = (long long)Cs * xsm;
          t1.split_out = h->x3;
          t1.bias = r.c1[dd].b;
          t1.tap_row0 = -(r.k * dl - dl) / 2;
          t1.dil = dl;
          t1.out = tmp;
          t1.epi = TCONV_SNAKE;
          t1.alpha = r.a2 + dd * Cs;
          t1.inv = r.i2 + dd * Cs;
          H_TRY(launch_tconv(t1, st));
          TConvArgs t2 = t;
          t2.A = tmp;
          t2.W = h->x3 ? r.c2[dd].Ws : r.c2[dd].W;
          t2.bias = r.c2[dd].b;
          t2.tap_row0 = -(r.k - 1) / 2;
          t2.out = xr;
          if (dd == 0) t2.resid_in = base;
          t2.epi = TCONV_RESID;
          if (dd < 2) {
            t2.alpha = r.a1 + (dd + 1) * Cs;
            t2.inv = r.i1 + (dd + 1) * Cs;
            t2.out2 = a_in;
            t2.split_out2 = h->x3;
            t2.ldo2 = (long long)Cs * xsm;
          }
          H_TRY(launch_tconv(t2, st));
          continue;
        }
        ConvGeo c1 = geo(r.c1[dd], vs, pl.vs_s[s][n], ss, ls, ss, a_in, tmp, HE_SNAKE);
        c1.dil = dl;
        c1.off = -(r.k * dl - dl) / 2;
        c1.alpha = r.a2 + dd * Cs;
        c1.inv = r.i2 + dd * Cs;
        H_TRY(run(c1));
        ConvGeo c2 = geo(r.c2[dd], vs, pl.vs_s[s][n], ss, ls, ss, tmp, xr, HE_RESID);
        c2.off = -(r.k - 1) / 2;
        if (dd == 0) c2.resid = base;
        if (dd < 2) {
          c2.alpha = r.a1 + (dd + 1) * Cs;
          c2.inv = r.i1 + (dd + 1) * Cs;
          c2.out2 = a_in;
        }
        H_TRY(run(c2));
      }
      return T2W_OK;
    };
    rc = resblock(g.src, sd, ta, reinterpret_cast<float*>(P(o_ar[s][0])), nullptr, src_tc);  // ar[0]: scratch
    if (!rc) rc = ck(cudaEventRecord(h->join_ev, st));
    st = st_main;
    if (rc) return fail(rc);
    rc = ck(cudaStreamWaitEvent(st, h->join_ev, 0));  // the fan-out below reads sd and reuses ar[0]
    if (rc) return fail(rc);
    forked = false;
    float* xr[3] = {reinterpret_cast<float*>(P(o_xr[s][0])), reinterpret_cast<float*>(P(o_xr[s][1])),
                    reinterpret_cast<float*>(P(o_xr[s][2]))};
    float* ar[3] = {reinterpret_cast<float*>(P(o_ar[s][0])), reinterpret_cast<float*>(P(o_ar[s][1])),
                    reinterpret_cast<float*>(P(o_ar[s][2]))};
    // xs += source branch (the three ResBlocks' common input, in place), with each block's first Snake of it
    Snake3 sn;
    for (int j = 0; j < 3; ++j) {
      sn.al[j] = g.res[j].a1;
      sn.inv[j] = g.res[j].i1;
    }
    rc = ck(launch_k(k_fanout, dim3(grid_for(nel / 4)), dim3(256), 0, st, (const float*)xs, (const float*)sd, nel, Cs,
                     h->x3, res_tc ? 1 : 0, xs, ar[0], ar[1], ar[2], sn));
    if (rc) return fail(rc);
    // the three ResBlocks read xs and write their own streams: ResBlocks 1 and 2 run on streams of their own, beside
    // ResBlock 0, each with scratch of its own (at small batches a ResBlock's convs cover few row tiles)
    rc = ck(cudaEventRecord(h->fork_ev, st));
    for (int k = 0; k < 2 && !rc; ++k) rc = ck(cudaStreamWaitEvent(h->res_st[k], h->fork_ev, 0));
    if (rc) return fail(rc);
    res_forked = true;
    for (int j = 0; j < 3; ++j) {
      float* tmp = j > 0 ? reinterpret_cast<float*>(P(o_tx[s][j - 1])) : ta;
      if (j > 0) st = h->res_st[j - 1];
      rc = resblock(g.res[j], xr[j], ar[j], tmp, xs, res_tc);
      if (!rc && j > 0) rc = ck(cudaEventRecord(h->res_ev[j - 1], st));
      st = st_main;
      if (rc) return fail(rc);
    }
    for (int k = 0; k < 2 && !rc; ++k) rc = ck(cudaStreamWaitEvent(st, h->res_ev[k], 0));  // the average reads all three
    if (rc) return fail(rc);
    res_forked = false;
    // the stage's output (x0 + x1 + x2) / 3 with the activation in front of what reads it: leaky_relu(., 0.1) before
    // the next stage's transposed conv, leaky_relu(., 0.01) before conv_post
    // conv_post on the tensor cores, and every transposed conv of the fp32 tensor-core mode, read [hi | lo] pairs
    const int split = (s == 2 && h->post_tc) || (s < 2 && h->x3);
    float* nx = reinterpret_cast<float*>(P(split ? o_xps : o_sd[s]));
    rc = ck(launch_k(k_avg3, dim3(grid_for(nel / 4)), dim3(256), 0, st, (const float*)xr[0], (const float*)xr[1],
                     (const float*)xr[2], nel, Cs, split, s < 2 ? c.lrelu_slope : 0.01f, nx));
    if (rc) return fail(rc);
    x = nx;
    vin = vs;
    s_in = ss;
    l_in = ls;
    nvin = pl.vs_s[s][n];
  }
  // 7. conv_post, inverse STFT, cross-fade, output, caches
  float* post = reinterpret_cast<float*>(P(o_post));
  {
    const int* ss2 = reinterpret_cast<const int*>(P(o_ss[2]));
    const int* ls2 = reinterpret_cast<const int*>(P(o_ls[2]));
    if (h->post_tc) {
      const int cin = C0 >> 3;
      TConvArgs t;
      t.A = x;
      t.lda = 2 * cin;
      t.rows_a = pl.A[3];
      t.W = h->post_ws;
      t.bias = h->post_bs;
      t.M = pl.A[3];
      t.N = 32;
      t.Cin = cin;
      t.taps = h->post.k;
      t.tap_row0 = -(h->post.k / 2);
      t.out = post;
      t.ldo = post_ld;
      t.pad = reinterpret_cast<const uint8_t*>(P(o_pad[3]));
      t.split_in = 1;
      t.err = h->err;
      rc = launch_tconv(t, st);
    } else {
      rc = run(geo(h->post, reinterpret_cast<const int*>(P(o_vs[2])), pl.vs_s[2][n], ss2, ls2, ss2, x, post,
                   HE_NONE));
    }
    if (rc) return fail(rc);
  }
  {
    dim3 grid((480 * h->max_frames + kIstftChunk - 1) / kIstftChunk, n);
    rc = ck(launch_k(k_istft_out, grid, dim3(256), 0, st, (const float*)post, post_ld, drows, (const float*)h->tw,
                     (const double*)h->hamming, c.audio_limit, 480.f, speech, (const float*)h->cache, h->cache_ld,
                     kMelCache * c.mel + kSrcCache, out_samples));
    if (rc) return fail(rc);
    rc = ck(launch_k(k_hift_caches, dim3(n), dim3(256), 0, st, drows, (const float*)mel, c.mel, (const float*)src,
                     (const float*)speech, h->cache, h->cache_ld, 0, kMelCache * c.mel, kMelCache * c.mel + kSrcCache,
                     480.f));
    if (rc) return fail(rc);
  }
  return T2W_OK;
  };
  int rc = T2W_OK;
  if (capture) {
    if (!h->cap_stream) rc = cudaStreamCreateWithFlags(&h->cap_stream, cudaStreamNonBlocking) ? T2W_ERR_CUDA : T2W_OK;
    if (!rc) rc = cudaStreamBeginCapture(h->cap_stream, cudaStreamCaptureModeThreadLocal) ? T2W_ERR_CUDA : T2W_OK;
    if (!rc) {
      const int re = enqueue(h->cap_stream);
      cudaGraph_t gr = nullptr;
      const cudaError_t ec = cudaStreamEndCapture(h->cap_stream, &gr);
      rc = re ? re : (ec != cudaSuccess ? T2W_ERR_CUDA : T2W_OK);
      if (!rc && cudaGraphInstantiate(&hg->exec, gr, 0) != cudaSuccess) rc = T2W_ERR_CUDA;
      if (gr) cudaGraphDestroy(gr);
    }
    if (rc) {
      drop_graph();
      return rc;
    }
    ++h->n_captures;
  }
  if (hg) {
    H_CUDA(cudaGraphLaunch(hg->exec, st));
    ++h->n_replays;
  } else {
    rc = enqueue(st);
    if (rc) {
      cudaFreeAsync(ws, st);
      return rc;
    }
    ++h->n_eager;
  }
  if (graph)
    H_CUDA(cudaMemcpyAsync(b->out, out_samples, (size_t)pl.out_samples * 4, cudaMemcpyDeviceToDevice, st));
  if (b->source) H_CUDA(cudaMemcpyAsync(b->source, src, (size_t)pl.samples * 4, cudaMemcpyDeviceToDevice, st));
  if (b->speech) H_CUDA(cudaMemcpyAsync(b->speech, speech, (size_t)pl.samples * 4, cudaMemcpyDeviceToDevice, st));
  if (hg)
    H_CUDA(cudaEventRecord(hg->done, st));
  else
    cudaFreeAsync(ws, st);
  for (int i = 0; i < n; ++i) h->row_first[b->handle[i]] = 0;
  return T2W_OK;
}

int t2w_hift_counts(const t2w_hift* h, int64_t* replays, int64_t* captures, int64_t* eager) {
  if (!h) return T2W_ERR_INVALID;
  if (replays) *replays = h->n_replays;
  if (captures) *captures = h->n_captures;
  if (eager) *eager = h->n_eager;
  return T2W_OK;
}

int t2w_test_tconv(const t2w_tconv_args* a, void* stream) {
  if (!a) return T2W_ERR_INVALID;
  TConvArgs t;
  t.A = a->A;
  t.lda = a->lda;
  t.rows_a = a->rows_a;
  t.W = a->W;
  t.bias = a->bias;
  t.M = a->M;
  t.N = a->N;
  t.Cin = a->Cin;
  t.taps = a->taps;
  t.tap_row0 = a->tap_row0;
  t.dil = a->dil;
  t.out = a->out;
  t.ldo = a->ldo;
  t.row_mul = a->row_mul;
  t.row_add = a->row_add;
  t.pad = a->pad;
  t.epi = a->epi;
  t.alpha = a->alpha;
  t.inv = a->inv;
  t.out2 = a->out2;
  t.split_in = a->split_in;
  t.split_out = a->split_out;
  t.err = a->err;
  t.resid_in = a->resid_in;
  return launch_tconv(t, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
