// tcgen05 / TMEM GEMM for the DiT projections: C[M, N] = sum_tap A[m + tap_row0 + tap, :] . W[n, tap-block]^T.
//
// One persistent CTA per SM, 6 warps:
//   warp 0  : TMA producer (one elected lane), STAGES-deep ring of A [128 x 64] and W [BN x 64] bf16 tiles, 128B swizzle
//   warp 1  : TMEM allocator + single-thread tcgen05.mma issuer (M = 128, N = BN, K = 16 per instruction)
//   warps 2-9: epilogue in two halves of four warps; warp w reads TMEM lanes 32 (w % 4) .. +31, so each thread owns one
//              output row, and half (w - 2) / 4 takes every other 128-byte output box of the tile
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so a tile's epilogue overlaps the next tile's MMAs.
// Each epilogue half stages its boxes (128 rows x 128 bytes, 128B swizzle) in its own shared-memory slot and writes them
// with asynchronous TMA stores issued by the half's leader thread.  Two warps per SM sub-partition keep the TMEM loads
// and the epilogue math of one box overlapped with the other's.
// The causal convolutions use taps = 3, tap_row0 = -2: tap t of output row m reads activation row m - 2 + t, so the
// im2col matrix is never materialised; rows before 0 come back zero from TMA.  No TMA multicast.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16 elements per 128-byte swizzle row
constexpr int kMaxSmem = 232448;
constexpr int kBoxBytes = kBM * 128;  // one staged output box: 128 rows x 128 bytes

__host__ __device__ constexpr bool epi_f32_out(int epi) { return epi == T2W_EPI_F32; }

template <int BN, int EPI, bool TMA_OUT>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_ELEM = epi_f32_out(EPI) ? 4 : 2;
  static constexpr int BOX_COLS = 128 / OUT_ELEM;
  static constexpr int N_BOXES = TMA_OUT ? BN / BOX_COLS : 0;
  static constexpr int OUT_BYTES = TMA_OUT ? 2 * kBoxBytes : 0;  // one staging slot per epilogue half
  static constexpr int FIXED = 1024 + 256;
  static constexpr int STAGES_FIT = (kMaxSmem - FIXED - OUT_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_BYTES + FIXED;
  static constexpr int THREADS = 320;
  static_assert(STAGES >= 2, "not enough shared memory for a 2-stage ring");
  static_assert(B_BYTES % 1024 == 0, "W tile must keep 1024-byte alignment of the swizzle atoms");
  static_assert(!TMA_OUT || (BN % BOX_COLS == 0 && N_BOXES % 2 == 0), "output tile must be an even number of boxes");
};

struct DevArgs {
  int M, N, K, taps, tap_row0, tiles_n, num_tiles;
  const float* bias;
  void* out;
  int ldo;
  const float* qn_w;
  const float* qn_b;
  const float* kn_w;
  const float* kn_b;
  float qk_eps;
  int* err;
};

T2W_DEV void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
T2W_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
T2W_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
T2W_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Named barrier of one epilogue half (ids 1 and 2, 128 threads each).
T2W_DEV void epi_barrier(int half) { asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory"); }

// 16-byte chunk `c` of row `r` inside one staged box (128B swizzle: chunk index XOR row % 8).
T2W_DEV uint8_t* box_chunk(uint8_t* box, int r, int c) { return box + r * 128 + ((c ^ (r & 7)) << 4); }

T2W_DEV void add_bias(float* v, const float* __restrict__ b, int n) {
#pragma unroll
  for (int j = 0; j < n / 4; ++j) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(b) + j);
    v[4 * j + 0] += q.x;
    v[4 * j + 1] += q.y;
    v[4 * j + 2] += q.z;
    v[4 * j + 3] += q.w;
  }
}

// Write 64 bf16 values (one row of one bf16 box) into the staging box.
T2W_DEV void stage_bf16_row(uint8_t* box, int r, const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    u.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    u.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    u.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(box_chunk(box, r, c)) = u;
  }
}

// Direct-store epilogue of one tile (BN = 80 final layer: no staging).
template <int BN, int EPI>
T2W_DEV void epilogue_direct(const DevArgs& p, uint32_t taddr, int row, int n0) {
  static_assert(EPI == T2W_EPI_F32 || EPI == T2W_EPI_BF16, "direct stores: f32 / bf16 only");
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    float v[16];
    tmem_ld16(taddr + c, v);
    if (row >= p.M) continue;
    add_bias(v, p.bias + n0 + c, 16);
    if constexpr (EPI == T2W_EPI_F32) {
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + n0 + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + n0 + c);
      dst[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
      dst[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                          pack_bf16x2(v[14], v[15]));
    }
  }
}

// Box b of a tile (BOX_COLS output columns of this thread's row r) into its staging box.
template <int EPI, int BOX_COLS>
T2W_DEV void epilogue_box(const DevArgs& p, uint32_t taddr, int r, int n0, int b, uint8_t* box) {
  if constexpr (EPI == T2W_EPI_F32) {
    float v[32];
    tmem_ld32(taddr + 32 * b, v);
    add_bias(v, p.bias + n0 + 32 * b, 32);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(box_chunk(box, r, c)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  } else {
    // bf16 outputs: a 64-column box (one head for the QKV epilogue)
    const int c0 = n0 + 64 * b;
    float v[64];
    tmem_ld32p(taddr + 64 * b, v);
    tmem_ld32p(taddr + 64 * b + 32, v + 32);
    add_bias(v, p.bias + c0, 64);
    if constexpr (EPI == T2W_EPI_QKV) {
      const int qcols = p.N / 3;
      if (c0 < 2 * qcols) {  // a q or k head: LayerNorm over its 64 values (affine), fp32
        const float* nw = c0 < qcols ? p.qn_w : p.kn_w;
        const float* nb = c0 < qcols ? p.qn_b : p.kn_b;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) s += v[i];
        const float mean = s * (1.f / 64.f);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float d = v[i] - mean;
          ss += d * d;
        }
        const float rstd = rsqrtf(ss * (1.f / 64.f) + p.qk_eps);
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          const float4 w4 = __ldg(reinterpret_cast<const float4*>(nw + i));
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(nb + i));
          v[i + 0] = fmaf((v[i + 0] - mean) * rstd, w4.x, b4.x);
          v[i + 1] = fmaf((v[i + 1] - mean) * rstd, w4.y, b4.y);
          v[i + 2] = fmaf((v[i + 2] - mean) * rstd, w4.z, b4.z);
          v[i + 3] = fmaf((v[i + 3] - mean) * rstd, w4.w, b4.w);
        }
      }
    } else if constexpr (EPI == T2W_EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = gelu_tanh(v[i]);
    }
    stage_bf16_row(box, r, v);
  }
}

template <int BN, int EPI, bool TMA_OUT>
__global__ void __launch_bounds__(320, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
           const __grid_constant__ CUtensorMap tmC, const DevArgs p) {
  using C = GemmCfg<BN, EPI, TMA_OUT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sOut = sB + C::STAGES * C::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::OUT_BYTES);
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
      mbar_init(&tempty[a], 8);  // one arrival per epilogue warp
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    if constexpr (TMA_OUT) tma_prefetch_desc(&tmC);
  }
  pdl_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch();
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
    const int half = (warp - 2) >> 2;
    const int r = q * 32 + lane;  // tile row == TMEM lane
    const bool leader = lane == 0 && q == 2;  // warps 2 and 6: store issuers of the two halves
    uint8_t* slot = sOut + half * kBoxBytes;
    // `ok` stays warp-uniform (tcgen05.ld is .sync.aligned); after a timed-out wait the warp skips all further waits
    // and work but still reaches every named barrier, so no warp is left waiting at one.
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], (it >> 1) & 1, p.err));
      if (ok) tc_fence_after();
      if constexpr (!TMA_OUT) {
        if (ok && half == 0) epilogue_direct<BN, EPI>(p, taddr, m0 + r, n0);
      } else {
#pragma unroll 1
        for (int b = half; b < C::N_BOXES; b += 2) {
          // this half's previous store has finished reading its slot
          if (leader) bulk_wait_read0();
          epi_barrier(half);
          if (ok) epilogue_box<EPI, C::BOX_COLS>(p, taddr, r, n0, b, slot);
          fence_proxy_async_smem();
          epi_barrier(half);
          if (leader && ok) {
            tma_store_2d(&tmC, slot, n0 + b * C::BOX_COLS, m0);
            bulk_commit();
          }
        }
      }
      if (ok) {  // every TMEM column this warp reads of the accumulator has been read
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
    }
    if constexpr (TMA_OUT) {
      if (leader) bulk_wait0();
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN, int EPI, bool TMA_OUT>
int launch_impl(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const WeightMaps* wm,
                const CUtensorMap* tmC) {
  const CUtensorMap* tmW = nullptr;
  if (wm) {
    tmW = BN == 80 ? (wm->has80 ? &wm->bn80 : nullptr) : BN == 128 ? (wm->has128 ? &wm->bn128 : nullptr)
                                                                 : (wm->has256 ? &wm->bn256 : nullptr);
    if (!tmW) return T2W_ERR_INVALID;
  }
  using C = GemmCfg<BN, EPI, TMA_OUT>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm<BN, EPI, TMA_OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
    attr_done = true;
  }
  CUtensorMap ma, mw, mc;
  if (!tmA) {
    if (!make_tmap_2d(&ma, a.A, 2, (uint64_t)a.rows_a, (uint64_t)a.K, (uint64_t)a.lda * 2, kBM, kBK)) return T2W_ERR_INVALID;
    tmA = &ma;
  }
  if (!tmW) {
    if (!make_tmap_2d(&mw, a.W, 2, (uint64_t)a.N, (uint64_t)a.K * a.taps, (uint64_t)a.K * a.taps * 2, BN, kBK))
      return T2W_ERR_INVALID;
    tmW = &mw;
  }
  if (!tmC) {
    if (TMA_OUT) {
      const bool f32 = epi_f32_out(EPI);
      if (!make_tmap_2d(&mc, a.out, f32 ? 4 : 2, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.ldo * (f32 ? 4 : 2), kBM,
                        C::BOX_COLS))
        return T2W_ERR_INVALID;
    } else {
      mc = *tmA;  // unused
    }
    tmC = &mc;
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
  p.qn_w = a.qn_w;
  p.qn_b = a.qn_b;
  p.kn_w = a.kn_w;
  p.kn_b = a.kn_b;
  p.qk_eps = a.qk_eps;
  p.err = a.err;
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  cudaError_t e = launch_k(k_gemm<BN, EPI, TMA_OUT>, dim3(grid), dim3(C::THREADS), C::SMEM, st, *tmA, *tmW, *tmC, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace

bool gemm_n_supported(int N) { return N == 80 || (N > 0 && N % 128 == 0); }

bool make_weight_maps(WeightMaps* m, const void* W, int N, int Ktot) {
  *m = WeightMaps();
  if (N == 80) return (m->has80 = make_tmap_2d(&m->bn80, W, 2, N, Ktot, (uint64_t)Ktot * 2, 80, kBK));
  if (N % 128) return false;
  m->has128 = make_tmap_2d(&m->bn128, W, 2, N, Ktot, (uint64_t)Ktot * 2, 128, kBK);
  if (N % 256 == 0) m->has256 = make_tmap_2d(&m->bn256, W, 2, N, Ktot, (uint64_t)Ktot * 2, 256, kBK);
  return m->has128;
}

// Column tile: 80 for the 80-wide final layer, else 256 (a 128 x 128 tile needs operand bytes from shared memory
// faster than the SM delivers them beside the TMA writes; 128 x 256 runs the tensor core at its rate), 128 only when N
// is not a multiple of 256.
int gemm_block_n_for(int N, int M, int epi) {
  (void)M;
  (void)epi;
  if (N == 80) return 80;
  if (N % 256 == 0) return 256;
  if (N % 128 == 0) return 128;
  return 0;
}

int launch_gemm(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const WeightMaps* tmW,
                const CUtensorMap* tmC) {
  if (!a.A || !a.W || !a.bias || !a.out || a.M <= 0 || a.M % kBM || a.K <= 0 || a.K % kBK || a.taps < 1 ||
      a.rows_a <= 0 || a.lda < a.K || a.lda % 8 || a.ldo % 8)
    return T2W_ERR_INVALID;
  const int bn = gemm_block_n_for(a.N, a.M, a.epi);
  if (!bn) return T2W_ERR_INVALID;
  if (a.epi == T2W_EPI_QKV && (a.N % 3 || (a.N / 3) % 64 || !a.qn_w || !a.qn_b || !a.kn_w || !a.kn_b)) return T2W_ERR_INVALID;
  if (bn == 80) {
    if (a.epi == T2W_EPI_F32) return launch_impl<80, T2W_EPI_F32, false>(a, st, tmA, tmW, tmC);
    if (a.epi == T2W_EPI_BF16) return launch_impl<80, T2W_EPI_BF16, false>(a, st, tmA, tmW, tmC);
    return T2W_ERR_INVALID;
  }
  if (bn == 256) {
    switch (a.epi) {
      case T2W_EPI_F32: return launch_impl<256, T2W_EPI_F32, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_BF16: return launch_impl<256, T2W_EPI_BF16, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_GELU: return launch_impl<256, T2W_EPI_GELU, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_QKV: return launch_impl<256, T2W_EPI_QKV, true>(a, st, tmA, tmW, tmC);
      default: return T2W_ERR_INVALID;
    }
  }
  switch (a.epi) {
    case T2W_EPI_F32: return launch_impl<128, T2W_EPI_F32, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_BF16: return launch_impl<128, T2W_EPI_BF16, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_GELU: return launch_impl<128, T2W_EPI_GELU, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_QKV: return launch_impl<128, T2W_EPI_QKV, true>(a, st, tmA, tmW, tmC);
    default: return T2W_ERR_INVALID;
  }
}

}  // namespace t2w
