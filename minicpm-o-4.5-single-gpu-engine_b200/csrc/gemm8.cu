// Block-scaled FP8 (e4m3) tcgen05 GEMM for the DiT projections of the FP8 path:
//   C[M, N] = sum_tap (A8[m + tap_row0 + tap, :] * 2^sfA) . (W8[n, tap-block] * 2^sfW)^T   (+ epilogue)
// A8 and W8 hold e4m3 values; every 32-element K block of every row of either operand has its own UE8M0 scale byte
// (the weights repeat one scale over the four 32-blocks of each 1 x 128 block).  The tensor core applies the scales
// (kind::mxf8f6f4.block_scale), so the fp32 accumulator is the dequantised product and the epilogues are those of the
// bf16 GEMM.  This is the FP8 weight path of the reference's fp8 linear (engine/runtime/fp8.py:1-40: e4m3 weights,
// per-token-scaled e4m3 activations, fp32 accumulation), with per-block instead of per-row scales.
//
// One persistent CTA per SM, 10 warps:
//   warp 0  : producer: TMA tiles of A [128 x 128 B] and W [256 x 128 B] (128B swizzle) plus the stage's scale-factor
//             atoms (bulk copies: 512 B for A's 128 rows, 1 KB for W's 256 rows), 3 stages
//   warp 1  : TMEM allocator + MMA issuer: per stage, tcgen05.cp of the atoms into TMEM, then 4 MMAs of K = 32
//   warps 2-9: epilogue (as the bf16 GEMM): each warp loads both of its 64-column boxes of the accumulator, releases
//             TMEM, then finishes and stores them with per-warp TMA stores
// The accumulator is single-buffered (256 columns; the scale factors take TMEM columns 256-291), and released as soon
// as every epilogue warp holds its part in registers.
//
// Scale-factor atoms (also the layout the quantisers write): for a [rows, C] e4m3 matrix, one 512-byte atom per
// (128-row tile, 128-column block); row r of the tile at byte (r % 32) * 16 + (r / 32) * 4, its 32-column block
// j % 4 at +j % 4 (sf_offset()).  tcgen05.cp 32x128b.warpx4 moves an atom into 4 TMEM columns of all 128 lanes.
// Row-shifted operands (the causal conv's taps read rows m - 2 + t) use atoms written with the rows shifted by
// d = -(tap_row0 + tap): layout d holds row x at position x + d, so every tap reads whole atoms.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 128;  // kBK e4m3 elements = 128 bytes = one swizzle row
constexpr int kStages = 3;
constexpr int kABytes = kBM * kBK, kBBytes = kBN * kBK;
constexpr int kSfABytes = 512, kSfBBytes = 1024;
constexpr int kStRows = 32, kSlotBytes = kStRows * 128, kEpiWarps = 8;
constexpr int kSmem = 1024 + kStages * (kABytes + kBBytes + kSfABytes + kSfBBytes) + kEpiWarps * kSlotBytes + 256;
static_assert((kStages * (kABytes + kBBytes)) % 1024 == 0, "output slots must start on a 1024-byte boundary");
constexpr int kTmemCols = 512;
constexpr uint32_t kSfCol0 = 256, kSfColsPerStage = 12;  // A: 4 columns, B: 8 columns

struct DevArgs {
  int M, N, K, taps, tap_row0, tiles_n, num_tiles, rows_a;
  const uint8_t* sfa;        // layout 0 of A's scale atoms
  long long sfa_layout;      // bytes between layouts d and d + 1
  const uint8_t* sfw;        // W's atoms: [k block of 128][N / 128][512]
  const float* bias;
  void* out;                 // bf16 [M, ldo] (or e4m3 for the GELU epilogue)
  int ldo;
  uint8_t* out_sf;           // GELU epilogue: the output's scale atoms (layout 0)
  const float* qn_w;
  const float* qn_b;
  const float* kn_w;
  const float* kn_b;
  float qk_eps;
  int* err;
  const void* pf;  // L2 prefetch of the next GEMM's weights (see Gemm8Args)
  unsigned pf_bytes;
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
T2W_DEV uint8_t* box_chunk(uint8_t* box, int r, int c) { return box + r * 128 + ((c ^ (r & 7)) << 4); }
T2W_DEV float2 u2f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }
T2W_DEV float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }

// Bias, the epilogue's own math, and (bf16 outputs) the packed words of one 64-column box of this thread's row.
template <int EPI>
T2W_DEV void box_math(const DevArgs& p, int c0, const uint32_t* raw, float2 (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = add2(u2f2(raw[2 * i], raw[2 * i + 1]), ldg2(p.bias + c0 + 2 * i));
  if constexpr (EPI == T2W_EPI_QKV) {
    const int qcols = p.N / 3;
    if (c0 < 2 * qcols) {  // a q or k head: LayerNorm over its 64 values (affine), fp32, two passes
      const float* nw = c0 < qcols ? p.qn_w : p.kn_w;
      const float* nb = c0 < qcols ? p.qn_b : p.kn_b;
      float2 s[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
      for (int i = 4; i < 32; ++i) s[i & 3] = add2(s[i & 3], v[i]);
      const float2 s2 = add2(add2(s[0], s[1]), add2(s[2], s[3]));
      const float mean = (s2.x + s2.y) * (1.f / 64.f);
      const float2 nm = make_float2(-mean, -mean);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = add2(v[i], nm);
      float2 q[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < 32; ++i) q[i & 3] = fma2(v[i], v[i], q[i & 3]);
      const float2 q2 = add2(add2(q[0], q[1]), add2(q[2], q[3]));
      const float rstd = rsqrtf((q2.x + q2.y) * (1.f / 64.f) + p.qk_eps);
      const float2 rs = make_float2(rstd, rstd), zero = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fma2(fma2(v[i], rs, zero), ldg2(nw + 2 * i), ldg2(nb + 2 * i));
    }
  } else if constexpr (EPI == T2W_EPI_GELU_FP8) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = make_float2(gelu_tanh(v[i].x), gelu_tanh(v[i].y));
  }
}

template <int EPI>
__global__ void __launch_bounds__(320, 1)
    k_gemm8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
            const __grid_constant__ CUtensorMap tmC, const DevArgs p) {
  constexpr bool kFp8Out = EPI == T2W_EPI_GELU_FP8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // operand tiles and output slots first: every swizzled buffer starts on a 1024-byte boundary (the 128B swizzle
  // pattern is a function of the shared-memory address bits 7-9)
  uint8_t* sA = smem;
  uint8_t* sB = sA + kStages * kABytes;
  uint8_t* sOut = sB + kStages * kBBytes;
  uint8_t* sSfA = sOut + kEpiWarps * kSlotBytes;
  uint8_t* sSfB = sSfA + kStages * kSfABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSfB + kStages * kSfBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kEpiWarps);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmC);
  }
  pdl_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch();
  const uint32_t tmem = *tmem_slot;

  const int kb_per_tap = p.K / kBK;
  const int num_kb = kb_per_tap * p.taps;
  const int kblocks_a = p.K / kBK;  // 128-column blocks of A: its atoms per 128-row tile

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * kBN;
        if (tile + (int)gridDim.x >= p.num_tiles) prefetch_l2_piece(p.pf, p.pf_bytes, blockIdx.x);  // last tile
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&empty[stage], phase ^ 1u, p.err))) break;
          mbar_expect_tx(&full[stage], kABytes + kBBytes + kSfABytes + kSfBBytes);
          const int tap = kb / kb_per_tap, kk = (kb - tap * kb_per_tap) * kBK;
          tma_load_2d(sA + stage * kABytes, &tmA, kk, m0 + p.tap_row0 + tap, &full[stage]);
          tma_load_2d(sB + stage * kBBytes, &tmW, tap * p.K + kk, n0, &full[stage]);
          const int d = -(p.tap_row0 + tap);  // the atom layout whose tiles start at row m0 + tap_row0 + tap
          bulk_load(sSfA + stage * kSfABytes,
                    p.sfa + d * p.sfa_layout + ((long long)(m0 / kBM) * kblocks_a + kk / kBK) * kSfABytes, kSfABytes,
                    &full[stage]);
          bulk_load(sSfB + stage * kSfBBytes,
                    p.sfw + ((long long)kb * (p.N / 128) + n0 / 128) * 512, kSfBBytes, &full[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
        if (!(ok = mbar_wait(tempty, (it & 1) ^ 1u, p.err))) break;
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, p.err))) break;
          tc_fence_after();
          const uint32_t sfa_t = tmem + kSfCol0 + kSfColsPerStage * stage, sfb_t = sfa_t + 4;
          tmem_cp_32x128b_x4(sfa_t, sdesc_noswz(smem_u32(sSfA + stage * kSfABytes), 128, 128));
          tmem_cp_32x128b_x4(sfb_t, sdesc_noswz(smem_u32(sSfB + stage * kSfBBytes), 128, 128));
          tmem_cp_32x128b_x4(sfb_t + 4, sdesc_noswz(smem_u32(sSfB + stage * kSfBBytes + 512), 128, 128));
          const uint32_t a0 = smem_u32(sA + stage * kABytes), b0 = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            umma_mxf8(tmem, sdesc_sw128(a0 + 32 * k, 1024, 16), sdesc_sw128(b0 + 32 * k, 1024, 16),
                      idesc_mxf8(kBM, kBN, (uint32_t)k), sfa_t, sfb_t, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(tfull);
      }
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    uint8_t* slot = sOut + (warp - 2) * kSlotBytes;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * kBN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
      if (!__all_sync(0xffffffffu, mbar_wait(tfull, it & 1, p.err))) break;
      tc_fence_after();
      // both of this warp's boxes (columns 64 b, b = half, half + 2) into registers, then hand the accumulator back
      uint32_t raw[2][64];
      tmem_ld64_nowait(taddr + 64 * half, raw[0]);
      tmem_ld64_nowait(taddr + 64 * (half + 2), raw[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
#pragma unroll
      for (int bi = 0; bi < 2; ++bi) {
        const int b = half + 2 * bi;
        const int c0 = n0 + 64 * b;
        float2 v[32];
        box_math<EPI>(p, c0, raw[bi], v);
        uint32_t w[32];
        if constexpr (kFp8Out) {
          // two 32-column blocks, each with its own power-of-two scale -> 64 e4m3 bytes
          uint32_t e2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(v[16 * h + i].x), fabsf(v[16 * h + i].y)));
            e2[h] = ue8m0_for_amax(amax);
            const float inv = ue8m0_inv(e2[h]);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              w[8 * h + i] = e4m3x4(v[16 * h + 2 * i].x * inv, v[16 * h + 2 * i].y * inv, v[16 * h + 2 * i + 1].x * inv,
                                    v[16 * h + 2 * i + 1].y * inv);
          }
          *reinterpret_cast<uint16_t*>(p.out_sf + sf_offset(m0 + r, c0 / 32, p.N)) = (uint16_t)(e2[0] | (e2[1] << 8));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = pack_bf16x2(v[i].x, v[i].y);
        }
        // this warp's previous store has finished reading the slot
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        if constexpr (kFp8Out) {  // 32 rows x 64 bytes, 64-byte swizzle
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(slot + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        } else {  // 32 rows x 128 bytes, 128-byte swizzle
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(box_chunk(slot, lane, c)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, slot, c0, m0 + q * kStRows);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait0();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int EPI>
int launch8_impl(const Gemm8Args& a, cudaStream_t st, const CUtensorMap* tmA, const CUtensorMap* tmW,
                 const CUtensorMap* tmC) {
  static std::atomic<uint64_t> attr_done{0};
  {
    const cudaError_t e = smem_attr_once(k_gemm8<EPI>, kSmem, attr_done);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
  }
  CUtensorMap ma, mw, mc;
  if (!tmA) {
    if (!make_tmap_2d(&ma, a.A8, 1, (uint64_t)a.rows_a, (uint64_t)a.K, (uint64_t)a.lda, kBM, kBK)) return T2W_ERR_INVALID;
    tmA = &ma;
  }
  if (!tmW) {
    if (!make_tmap_2d(&mw, a.W8, 1, (uint64_t)a.N, (uint64_t)a.K * a.taps, (uint64_t)a.K * a.taps, kBN, kBK))
      return T2W_ERR_INVALID;
    tmW = &mw;
  }
  if (!tmC) {
    const bool ok = EPI == T2W_EPI_GELU_FP8
                        ? make_tmap_2d_ex(&mc, a.out, 1, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.ldo, kStRows, 64, 64)
                        : make_tmap_2d(&mc, a.out, 2, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.ldo * 2, kStRows, 64);
    if (!ok) return T2W_ERR_INVALID;
    tmC = &mc;
  }
  DevArgs p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.taps = a.taps;
  p.tap_row0 = a.tap_row0;
  p.tiles_n = a.N / kBN;
  p.num_tiles = (a.M / kBM) * p.tiles_n;
  p.rows_a = a.rows_a;
  p.sfa = a.sfa;
  p.sfa_layout = a.sfa_layout;
  p.sfw = a.sfw;
  p.bias = a.bias;
  p.out = a.out;
  p.ldo = a.ldo;
  p.out_sf = a.out_sf;
  p.qn_w = a.qn_w;
  p.qn_b = a.qn_b;
  p.kn_w = a.kn_w;
  p.kn_b = a.kn_b;
  p.qk_eps = a.qk_eps;
  p.err = a.err;
  p.pf = a.pf;
  p.pf_bytes = a.pf_bytes;
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  cudaError_t e = launch_k(k_gemm8<EPI>, dim3(grid), dim3(320), kSmem, st, *tmA, *tmW, *tmC, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace

size_t gemm8_sf_bytes(int rows, int cols) { return (size_t)((rows + 127) / 128) * (cols / 128) * 512; }

int launch_gemm8(const Gemm8Args& a, cudaStream_t st, const CUtensorMap* tmA, const CUtensorMap* tmW,
                 const CUtensorMap* tmC) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a.A8 || !a.W8 || !a.sfa || !a.sfw || !a.bias || !a.out || a.M <= 0 || a.M % kBM || a.N <= 0 || a.N % kBN ||
      a.K <= 0 || a.K % kBK || a.taps < 1 || a.rows_a <= 0 || a.lda < a.K || a.lda % 16 || a.ldo % 16 ||
      !al16(a.sfa) || !al16(a.sfw) || a.sfa_layout % 16 || a.sfa_layouts < 1)
    return T2W_ERR_INVALID;
  // every tap's row shift d = -(tap_row0 + tap) needs its atom layout
  if (-a.tap_row0 > a.sfa_layouts - 1 || -(a.tap_row0 + a.taps - 1) < 0) return T2W_ERR_INVALID;
  switch (a.epi) {
    case T2W_EPI_BF16: return launch8_impl<T2W_EPI_BF16>(a, st, tmA, tmW, tmC);
    case T2W_EPI_QKV:
      if (a.N % 3 || (a.N / 3) % 64 || !a.qn_w || !a.qn_b || !a.kn_w || !a.kn_b) return T2W_ERR_INVALID;
      return launch8_impl<T2W_EPI_QKV>(a, st, tmA, tmW, tmC);
    case T2W_EPI_GELU_FP8:
      if (!a.out_sf || !al16(a.out_sf)) return T2W_ERR_INVALID;
      return launch8_impl<T2W_EPI_GELU_FP8>(a, st, tmA, tmW, tmC);
    default: return T2W_ERR_INVALID;
  }
}

}  // namespace t2w
