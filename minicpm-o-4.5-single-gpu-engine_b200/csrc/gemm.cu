// tcgen05 / TMEM GEMM for the DiT projections: C[M, N] = sum_tap A[m + tap_row0 + tap, :] . W[n, tap-block]^T.
//
// One persistent CTA per SM, 6 warps:
//   warp 0  : TMA producer (one elected lane), STAGES-deep ring of A [128 x 64] and W [BN x 64] bf16 tiles, 128B swizzle
//   warp 1  : TMEM allocator + single-thread tcgen05.mma issuer (M = 128, N = BN, K = 16 per instruction)
//   warps 2-5: epilogue; warp w reads TMEM lanes 32 (w % 4) .. +31, so each thread owns one output row
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so a tile's epilogue overlaps the next tile's MMAs.
// The causal convolutions use taps = 3, tap_row0 = -2: tap t of output row m reads activation row m - 2 + t, so the
// im2col matrix is never materialised; rows before 0 come back zero from TMA.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16 elements per 128-byte swizzle row

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN >= 256 ? 4 : 6;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(B_BYTES % 1024 == 0, "W tile must keep 1024-byte alignment of the swizzle atoms");
};

struct DevArgs {
  int M, N, K, taps, tap_row0, tiles_n, num_tiles;
  const float* bias;
  void* out;
  int ldo;
  float* resid;
  int ldr;
  const float* gate;
  const float* qn_w;
  const float* qn_b;
  const float* kn_w;
  const float* kn_b;
  float qk_eps;
  int* err;
};

T2W_DEV void store_bf16x16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 u0, u1;
  u0.x = pack_bf16x2(v[0], v[1]);
  u0.y = pack_bf16x2(v[2], v[3]);
  u0.z = pack_bf16x2(v[4], v[5]);
  u0.w = pack_bf16x2(v[6], v[7]);
  u1.x = pack_bf16x2(v[8], v[9]);
  u1.y = pack_bf16x2(v[10], v[11]);
  u1.z = pack_bf16x2(v[12], v[13]);
  u1.w = pack_bf16x2(v[14], v[15]);
  reinterpret_cast<uint4*>(dst)[0] = u0;
  reinterpret_cast<uint4*>(dst)[1] = u1;
}

T2W_DEV void add_vec16(float (&v)[16], const float* __restrict__ b) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(b) + j);
    v[4 * j + 0] += q.x;
    v[4 * j + 1] += q.y;
    v[4 * j + 2] += q.z;
    v[4 * j + 3] += q.w;
  }
}

template <int BN, int EPI>
T2W_DEV void epilogue(const DevArgs& p, uint32_t taddr, int row, int n0) {
  const bool row_ok = row < p.M;
  if constexpr (EPI == T2W_EPI_QKV) {
    const int qcols = p.N / 3;
#pragma unroll 1
    for (int g = 0; g < BN / 64; ++g) {
      const int c0 = n0 + g * 64;
      float v[4][16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tmem_ld16(taddr + g * 64 + 16 * j, v[j]);
        add_vec16(v[j], p.bias + c0 + 16 * j);
      }
      if (c0 < 2 * qcols) {  // q or k head: LayerNorm over the head's 64 values (affine), fp32
        const int d0 = (c0 % qcols) % 64;  // always 0: heads are 64-aligned inside the q / k blocks
        const float* nw = (c0 < qcols ? p.qn_w : p.kn_w) + d0;
        const float* nb = (c0 < qcols ? p.qn_b : p.kn_b) + d0;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int i = 0; i < 16; ++i) s += v[j][i];
        const float mean = s * (1.f / 64.f);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float d = v[j][i] - mean;
            ss += d * d;
          }
        const float rstd = rsqrtf(ss * (1.f / 64.f) + p.qk_eps);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int i = 0; i < 16; ++i) v[j][i] = (v[j][i] - mean) * rstd * __ldg(nw + 16 * j + i) + __ldg(nb + 16 * j + i);
      }
      if (row_ok) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + c0;
#pragma unroll
        for (int j = 0; j < 4; ++j) store_bf16x16(dst + 16 * j, v[j]);
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      const int col = n0 + c;
      float v[16];
      tmem_ld16(taddr + c, v);
      if (!row_ok) continue;
      add_vec16(v, p.bias + col);
      if constexpr (EPI == T2W_EPI_F32) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else if constexpr (EPI == T2W_EPI_BF16 || EPI == T2W_EPI_GELU) {
        if constexpr (EPI == T2W_EPI_GELU) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = gelu_tanh(v[i]);
        }
        store_bf16x16(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + col, v);
      } else if constexpr (EPI == T2W_EPI_RESID) {
        float4* r = reinterpret_cast<float4*>(p.resid + (size_t)row * p.ldr + col);
        const float4* g = reinterpret_cast<const float4*>(p.gate + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float4 x = r[j];
          const float4 gg = __ldg(g + j);
          x.x = fmaf(gg.x, v[4 * j + 0], x.x);
          x.y = fmaf(gg.y, v[4 * j + 1], x.y);
          x.z = fmaf(gg.z, v[4 * j + 2], x.z);
          x.w = fmaf(gg.w, v[4 * j + 3], x.w);
          r[j] = x;
        }
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const DevArgs p) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int kb_per_tap = p.K / kBK;
  const int num_kb = kb_per_tap * p.taps;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&empty[stage], phase ^ 1u, p.err))) break;
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          const int tap = kb / kb_per_tap, kk = (kb - tap * kb_per_tap) * kBK;
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, kk, m0 + p.tap_row0 + tap, &full[stage]);
          tma_load_2d(sB + stage * C::B_BYTES, &tmW, tap * p.K + kk, n0, &full[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!(ok = mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1u, p.err))) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, p.err))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES), b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_f16(d, sdesc_sw128(a0 + 32 * k, 1024, 16), sdesc_sw128(b0 + 32 * k, 1024, 16), idesc,
                     (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    const int q = warp & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, p.err)) break;
      tc_fence_after();
      const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      epilogue<BN, EPI>(p, taddr, m0 + q * 32 + lane, n0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN, int EPI>
int launch_impl(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const CUtensorMap* tmW) {
  using C = GemmCfg<BN>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
    attr_done = true;
  }
  CUtensorMap ma, mw;
  if (!tmA) {
    if (!make_tmap_2d(&ma, a.A, 2, (uint64_t)a.rows_a, (uint64_t)a.K * (a.taps == 1 ? 1 : 1), (uint64_t)a.lda * 2, kBM,
                      kBK))
      return T2W_ERR_INVALID;
    tmA = &ma;
  }
  if (!tmW) {
    if (!make_tmap_2d(&mw, a.W, 2, (uint64_t)a.N, (uint64_t)a.K * a.taps, (uint64_t)a.K * a.taps * 2, BN, kBK))
      return T2W_ERR_INVALID;
    tmW = &mw;
  }
  DevArgs p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.taps = a.taps;
  p.tap_row0 = a.tap_row0;
  p.tiles_n = a.N / BN;
  p.num_tiles = (a.M / kBM) * p.tiles_n;
  p.bias = a.bias;
  p.out = a.out;
  p.ldo = a.ldo;
  p.resid = a.resid;
  p.ldr = a.ldr;
  p.gate = a.gate;
  p.qn_w = a.qn_w;
  p.qn_b = a.qn_b;
  p.kn_w = a.kn_w;
  p.kn_b = a.kn_b;
  p.qk_eps = a.qk_eps;
  p.err = a.err;
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  k_gemm<BN, EPI><<<grid, 192, C::SMEM, st>>>(*tmA, *tmW, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

template <int BN>
int dispatch_epi(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const CUtensorMap* tmW) {
  switch (a.epi) {
    case T2W_EPI_F32: return launch_impl<BN, T2W_EPI_F32>(a, st, tmA, tmW);
    case T2W_EPI_BF16: return launch_impl<BN, T2W_EPI_BF16>(a, st, tmA, tmW);
    case T2W_EPI_GELU: return launch_impl<BN, T2W_EPI_GELU>(a, st, tmA, tmW);
    case T2W_EPI_RESID: return launch_impl<BN, T2W_EPI_RESID>(a, st, tmA, tmW);
    case T2W_EPI_QKV:
      if constexpr (BN % 64 == 0) return launch_impl<BN, T2W_EPI_QKV>(a, st, tmA, tmW);
      return T2W_ERR_INVALID;
    default: return T2W_ERR_INVALID;
  }
}

}  // namespace

int gemm_block_n(int N) {
  if (N % 256 == 0) return 256;
  if (N % 128 == 0) return 128;
  if (N == 80) return 80;
  return 0;
}

int launch_gemm(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const CUtensorMap* tmW) {
  if (!a.A || !a.W || !a.bias || a.M <= 0 || a.M % kBM || a.K <= 0 || a.K % kBK || a.taps < 1 || a.rows_a <= 0 ||
      a.lda < a.K || a.lda % 8)
    return T2W_ERR_INVALID;
  const int bn = gemm_block_n(a.N);
  if (!bn) return T2W_ERR_INVALID;
  if (a.epi == T2W_EPI_RESID && (!a.resid || !a.gate || a.ldr % 4)) return T2W_ERR_INVALID;
  if (a.epi != T2W_EPI_RESID && (!a.out || a.ldo % 8)) return T2W_ERR_INVALID;
  if (a.epi == T2W_EPI_QKV && (a.N % 3 || (a.N / 3) % 64 || !a.qn_w || !a.qn_b || !a.kn_w || !a.kn_b)) return T2W_ERR_INVALID;
  switch (bn) {
    case 256: return dispatch_epi<256>(a, st, tmA, tmW);
    case 128: return dispatch_epi<128>(a, st, tmA, tmW);
    case 80:
      if (a.epi == T2W_EPI_F32) return launch_impl<80, T2W_EPI_F32>(a, st, tmA, tmW);
      if (a.epi == T2W_EPI_BF16) return launch_impl<80, T2W_EPI_BF16>(a, st, tmA, tmW);
      return T2W_ERR_INVALID;
  }
  return T2W_ERR_INVALID;
}

}  // namespace t2w
