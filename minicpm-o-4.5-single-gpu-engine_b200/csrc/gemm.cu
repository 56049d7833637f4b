// tcgen05 / TMEM GEMM for the DiT projections: C[M, N] = sum_tap A[m + tap_row0 + tap, :] . W[n, tap-block]^T.
//
// One persistent CTA per SM, 10 warps:
//   warp 0  : TMA producer (one elected lane), STAGES-deep ring of A [128 x 64] and W [BN x 64] bf16 tiles, 128B swizzle
//   warp 1  : TMEM allocator + single-thread tcgen05.mma issuer (M = 128, N = BN, K = 16 per instruction)
//   warps 2-9: epilogue; warp w reads TMEM lanes 32 (w % 4) .. +31 (one output row per thread) and takes every other
//              128-byte output box of the tile, half (w - 2) / 4 the even or the odd ones
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so a tile's epilogue overlaps the next tile's MMAs,
// and each warp hands its accumulator columns back as soon as its last TMEM load of the tile has landed.  Every
// epilogue warp stages its 32 rows x 128 bytes of a box (128B swizzle) in a shared-memory slot of its own and writes
// them with an asynchronous TMA store from its lane 0, so the eight warps never wait for one another.
// The causal convolutions use taps = 3, tap_row0 = -2: tap t of output row m reads activation row m - 2 + t, so the
// im2col matrix is never materialised; rows before 0 come back zero from TMA.  No TMA multicast.
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16 elements per 128-byte swizzle row
constexpr int kMaxSmem = 232448;
constexpr int kStRows = 32;                // rows of one TMA store: one epilogue warp's TMEM lane quarter
constexpr int kSlotBytes = kStRows * 128;  // one warp's staging slot: 32 rows x 128 bytes
constexpr int kEpiWarps = 8;

__host__ __device__ constexpr bool epi_f32_out(int epi) { return epi == T2W_EPI_F32 || epi == T2W_EPI_RESID; }

template <int BN, int EPI, bool TMA_OUT>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_ELEM = epi_f32_out(EPI) ? 4 : 2;
  static constexpr int BOX_COLS = 128 / OUT_ELEM;
  static constexpr int N_BOXES = TMA_OUT ? BN / BOX_COLS : 0;
  static constexpr int OUT_BYTES = TMA_OUT ? kEpiWarps * kSlotBytes : 0;  // one staging slot per epilogue warp
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
  int* done_flags;  // per 128-row block: +1 from each epilogue warp once its stores of a tile are complete
  const float* gate;  // T2W_EPI_RESID: per-column gate of the residual update
  const void* pf;     // L2 prefetch of the next GEMM's weights (see GemmArgs)
  unsigned pf_bytes;
};

T2W_DEV void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
// out[box] += smem box (fp32 add performed in L2), evict-last: the residual stream it updates stays resident.
T2W_DEV void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::
          "l"(reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(smem_u32(smem_src)), "l"(policy)
      : "memory");
}
T2W_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
T2W_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
T2W_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 16-byte chunk `c` of row `r` inside one staged slot (128B swizzle: chunk index XOR row % 8).
T2W_DEV uint8_t* box_chunk(uint8_t* box, int r, int c) { return box + r * 128 + ((c ^ (r & 7)) << 4); }

// Direct-store epilogue of one tile (BN = 80 final layer: no staging).
template <int BN, int EPI>
T2W_DEV void epilogue_direct(const DevArgs& p, uint32_t taddr, int row, int n0) {
  static_assert(EPI == T2W_EPI_F32 || EPI == T2W_EPI_BF16, "direct stores: f32 / bf16 only");
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    float v[16];
    tmem_ld16(taddr + c, v);
    if (row >= p.M) continue;
    const float* b = p.bias + n0 + c;
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] += __ldg(b + j);
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

T2W_DEV float2 u2f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }
T2W_DEV float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }

// Epilogue math of box b for this thread's row: `raw` holds the box's accumulator columns (32 fp32 columns, or 64 for
// bf16 outputs); on return it holds the 32 words staged for the box (fp32 values, or bf16 pairs).
template <int EPI>
T2W_DEV void epilogue_math(const DevArgs& p, int n0, int b, uint32_t (&raw)[64]) {
  if constexpr (EPI == T2W_EPI_F32) {
    const float* bias = p.bias + n0 + 32 * b;
#pragma unroll
    for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(__uint_as_float(raw[i]) + __ldg(bias + i));
  } else if constexpr (EPI == T2W_EPI_RESID) {  // the update gate * (acc + bias); the TMA reduce adds it to out
    const float4* bias = reinterpret_cast<const float4*>(p.bias + n0 + 32 * b);
    const float4* gate = reinterpret_cast<const float4*>(p.gate + n0 + 32 * b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 bb = __ldg(bias + j), gg = __ldg(gate + j);
      raw[4 * j] = __float_as_uint(gg.x * (__uint_as_float(raw[4 * j]) + bb.x));
      raw[4 * j + 1] = __float_as_uint(gg.y * (__uint_as_float(raw[4 * j + 1]) + bb.y));
      raw[4 * j + 2] = __float_as_uint(gg.z * (__uint_as_float(raw[4 * j + 2]) + bb.z));
      raw[4 * j + 3] = __float_as_uint(gg.w * (__uint_as_float(raw[4 * j + 3]) + bb.w));
    }
  } else {
    const int c0 = n0 + 64 * b;
    float2 v[32];
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
    } else if constexpr (EPI == T2W_EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = make_float2(gelu_tanh(v[i].x), gelu_tanh(v[i].y));
    } else if constexpr (EPI == T2W_EPI_SILU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = make_float2(silu(v[i].x), silu(v[i].y));
    } else if constexpr (EPI == T2W_EPI_LEAKY) {
      const float slope = p.qk_eps;  // the leaky ReLU's negative slope travels in the q/k-norm eps field
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = make_float2(v[i].x > 0.f ? v[i].x : slope * v[i].x, v[i].y > 0.f ? v[i].y : slope * v[i].y);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) raw[i] = pack_bf16x2(v[i].x, v[i].y);
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
        if (tile + (int)gridDim.x >= p.num_tiles) prefetch_l2_piece(p.pf, p.pf_bytes, blockIdx.x);  // last tile
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
    uint8_t* slot = sOut + (warp - 2) * kSlotBytes;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      // warp-uniform (tcgen05.ld is .sync.aligned); after a timed-out wait the warp stops
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], (it >> 1) & 1, p.err))) break;
      tc_fence_after();
      if constexpr (!TMA_OUT) {
        if (half == 0) epilogue_direct<BN, EPI>(p, taddr, m0 + q * 32 + lane, n0);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
#pragma unroll 1
        for (int b = half; b < C::N_BOXES; b += 2) {
          uint32_t raw[64];
          if constexpr (epi_f32_out(EPI)) {
            float f[32];
            tmem_ld32(taddr + 32 * b, f);
#pragma unroll
            for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(f[i]);
          } else {
            tmem_ld64_nowait(taddr + 64 * b, raw);
            tmem_ld_wait();
          }
          if (b + 2 >= C::N_BOXES) {  // this warp's last TMEM load of the accumulator has landed
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
          epilogue_math<EPI>(p, n0, b, raw);
          // this warp's previous store has finished reading the slot
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(box_chunk(slot, lane, c)) =
                make_uint4(raw[4 * c], raw[4 * c + 1], raw[4 * c + 2], raw[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == T2W_EPI_RESID)
              tma_reduce_add_2d(&tmC, slot, n0 + b * C::BOX_COLS, m0 + q * kStRows, l2_policy_evict_last());
            else
              tma_store_2d(&tmC, slot, n0 + b * C::BOX_COLS, m0 + q * kStRows);
            bulk_commit();
          }
        }
        if (p.done_flags && lane == 0) {  // publish: this warp's rows of the tile are in global memory
          bulk_wait0();
          fence_proxy_async_global();
          __threadfence();
          red_release_add_gpu(p.done_flags + m0 / kBM, 1);
        }
      }
    }
    if constexpr (TMA_OUT) {
      if (lane == 0) bulk_wait0();
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------- CTA-pair variant (tcgen05 cta_group::2)
// A cluster of two CTAs on neighbouring SMs computes a 256 x 256 tile: CTA r of the pair loads rows 128 r .. + 127 of
// the tile's A and rows 128 r .. + 127 of its 256 W rows, and one M = 256 MMA issued by CTA 0 reads both CTAs' shared
// memory and accumulates each CTA's 128 output rows in that CTA's TMEM.  Per CTA and K block the operand bytes drop
// from 48 KB (128 x 256 single-CTA tile) to 32 KB for the same tensor work, which is what bounds the long-K GEMMs
// (their operands stream from L2).  Protocol (the CTA pair shares barrier offsets):
//   full[s]   CTA 0 only: arrive + expect the stage's bytes of both CTAs; both CTAs' TMA loads complete on it;
//   empty[s]  both CTAs: CTA 0's MMA commit arrives on the pair's empty[s] once the stage is consumed;
//   tfull[a]  both CTAs: CTA 0's commit after a tile's last MMA;
//   tempty[a] CTA 0 only: 16 arrivals (8 epilogue warps per CTA) once both CTAs hold the accumulator in registers.
// Both CTAs allocate TMEM with cta_group::2 from the same warp and free it after a cluster barrier.  No multicast load.
constexpr int kPairStages = 6;
constexpr int kPairABytes = kBM * kBK * 2, kPairBBytes = 128 * kBK * 2;
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
constexpr int kPairSmem = kPairStages * kPairStageBytes + kEpiWarps * kSlotBytes + 1024 + 256;

T2W_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `smem_addr`'s counterpart in CTA `rank` of the cluster.
T2W_DEV uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
T2W_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
T2W_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory that completes on an mbarrier of either CTA of the pair.
T2W_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y, uint32_t mbar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster_addr)
      : "memory");
}
T2W_DEV void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar`'s counterparts in both CTAs of the pair once this thread's issued MMAs have completed.
T2W_DEV void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"((unsigned short)3)
               : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(320, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmC, const DevArgs p) {
  constexpr int BN = 256;
  constexpr int BOX_COLS = epi_f32_out(EPI) ? 32 : 64;
  constexpr int N_BOXES = BN / BOX_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPairStages * kPairABytes;
  uint8_t* sOut = sB + kPairStages * kPairBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kEpiWarps * kSlotBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmC);
  }
  pdl_wait();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  pdl_launch();
  const uint32_t tmem = *tmem_slot;

  const int kb_per_tap = p.K / kBK;
  const int num_kb = kb_per_tap * p.taps;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {  // producer of this CTA's half of every stage
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += n_pairs) {
        const int m0 = (tile / p.tiles_n) * (2 * kBM) + (int)rank * kBM, n0 = (tile % p.tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&empty[stage], phase ^ 1u, p.err))) break;
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * kPairStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          const int tap = kb / kb_per_tap, kk = (kb - tap * kb_per_tap) * kBK;
          tma_load_2d_pair(sA + stage * kPairABytes, &tmA, kk, m0 + p.tap_row0 + tap, fb);
          tma_load_2d_pair(sB + stage * kPairBBytes, &tmW, tap * p.K + kk, n0 + (int)rank * 128, fb);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // the pair's MMA issuer
      constexpr uint32_t idesc = idesc_bf16(2 * kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = pair; tile < p.num_tiles && ok; tile += n_pairs, ++it) {
        const int acc = it & 1;
        if (!(ok = mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1u, p.err))) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, p.err))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * kPairABytes), b0 = smem_u32(sB + stage * kPairBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_pair(d, sdesc_sw128(a0 + 32 * k, 1024, 16), sdesc_sw128(b0 + 32 * k, 1024, 16), idesc,
                          (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage]);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair(&tfull[acc]);
      }
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* slot = sOut + (warp - 2) * kSlotBytes;
    int it = 0;
    for (int tile = pair; tile < p.num_tiles; tile += n_pairs, ++it) {
      const int acc = it & 1;
      const int m0 = (tile / p.tiles_n) * (2 * kBM) + (int)rank * kBM, n0 = (tile % p.tiles_n) * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], (it >> 1) & 1, p.err))) break;
      tc_fence_after();
#pragma unroll 1
      for (int b = half; b < N_BOXES; b += 2) {
        uint32_t raw[64];
        if constexpr (epi_f32_out(EPI)) {
          float f[32];
          tmem_ld32(taddr + 32 * b, f);
#pragma unroll
          for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(f[i]);
        } else {
          tmem_ld64_nowait(taddr + 64 * b, raw);
          tmem_ld_wait();
        }
        if (b + 2 >= N_BOXES) {  // this warp's last TMEM load of the accumulator: release it to the pair's issuer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&tempty[acc]), 0));
        }
        epilogue_math<EPI>(p, n0, b, raw);
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(box_chunk(slot, lane, c)) =
              make_uint4(raw[4 * c], raw[4 * c + 1], raw[4 * c + 2], raw[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (EPI == T2W_EPI_RESID)
            tma_reduce_add_2d(&tmC, slot, n0 + b * BOX_COLS, m0 + q * kStRows, l2_policy_evict_last());
          else
            tma_store_2d(&tmC, slot, n0 + b * BOX_COLS, m0 + q * kStRows);
          bulk_commit();
        }
      }
      if (p.done_flags && lane == 0 && m0 < p.M) {  // (CTA 1 of a pair past M when M % 256 == 128 stores nothing)
        bulk_wait0();
        fence_proxy_async_global();
        __threadfence();
        red_release_add_gpu(p.done_flags + m0 / kBM, 1);
      }
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs and TMEM loads are done in both CTAs
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
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
  static std::atomic<uint64_t> attr_done{0};
  {
    const cudaError_t e = smem_attr_once(k_gemm<BN, EPI, TMA_OUT>, C::SMEM, attr_done);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
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
      if (!make_tmap_2d(&mc, a.out, f32 ? 4 : 2, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.ldo * (f32 ? 4 : 2), kStRows,
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
  p.done_flags = TMA_OUT ? a.done_flags : nullptr;
  p.gate = a.gate;
  p.pf = a.pf;
  p.pf_bytes = a.pf_bytes;
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  cudaError_t e = launch_k(k_gemm<BN, EPI, TMA_OUT>, dim3(grid), dim3(C::THREADS), C::SMEM, st, *tmA, *tmW, *tmC, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}


// CTA-pair launch (cluster of 2): 256 x 256 tiles, grid of at most the pairs that can be resident at once.
template <int EPI>
int launch_pair_impl(const GemmArgs& a, cudaStream_t st, const CUtensorMap* tmA, const WeightMaps* wm,
                     const CUtensorMap* tmC) {
  static std::atomic<uint64_t> attr_done{0};
  {
    const cudaError_t e = smem_attr_once(k_gemm_pair<EPI>, kPairSmem, attr_done);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
  }
  static int max_pairs = -1;  // clusters resident at once (the same on every B200)
  if (max_pairs < 0) {
    cudaError_t e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(320);
    cfg.dynamicSmemBytes = kPairSmem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, k_gemm_pair<EPI>, &cfg);
    if (e != cudaSuccess || n <= 0) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
    max_pairs = n;
  }
  const CUtensorMap* tmW = (wm && wm->has128) ? &wm->bn128 : nullptr;
  CUtensorMap ma, mw, mc;
  if (!tmA) {
    if (!make_tmap_2d(&ma, a.A, 2, (uint64_t)a.rows_a, (uint64_t)a.K, (uint64_t)a.lda * 2, kBM, kBK)) return T2W_ERR_INVALID;
    tmA = &ma;
  }
  if (!tmW) {
    if (!make_tmap_2d(&mw, a.W, 2, (uint64_t)a.N, (uint64_t)a.K * a.taps, (uint64_t)a.K * a.taps * 2, 128, kBK))
      return T2W_ERR_INVALID;
    tmW = &mw;
  }
  if (!tmC) {
    const bool f32 = epi_f32_out(EPI);
    if (!make_tmap_2d(&mc, a.out, f32 ? 4 : 2, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.ldo * (f32 ? 4 : 2), kStRows,
                      f32 ? 32 : 64))
      return T2W_ERR_INVALID;
    tmC = &mc;
  }
  DevArgs p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.taps = a.taps;
  p.tap_row0 = a.tap_row0;
  p.tiles_n = a.N / 256;
  p.num_tiles = ((a.M + 2 * kBM - 1) / (2 * kBM)) * p.tiles_n;
  p.bias = a.bias;
  p.out = a.out;
  p.ldo = a.ldo;
  p.qn_w = a.qn_w;
  p.qn_b = a.qn_b;
  p.kn_w = a.kn_w;
  p.kn_b = a.kn_b;
  p.qk_eps = a.qk_eps;
  p.err = a.err;
  p.done_flags = a.done_flags;
  p.gate = a.gate;
  p.pf = nullptr;  // (the pair kernel issues no prefetch)
  p.pf_bytes = 0;
  const int pairs = p.num_tiles < max_pairs ? p.num_tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(320);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_pair<EPI>, *tmA, *tmW, *tmC, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

// Which 256-column GEMMs run on CTA pairs.  Measured on B200 (bf16, N = 512): the pair kernel wins on long K once
// there are several rounds of tiles (M = 44800: 3-tap conv 51.1 vs 54.5 us, K = 2048 75 vs 80 us), and loses on
// short K and on one-and-a-bit rounds (M = 11264), where the epilogue or the partial last round bounds the time.
// T2W_GEMM_PAIR=0 / =1 overrides the rule (never / always).
bool use_pair(const GemmArgs& a) {
  static int v = -2;
  if (v == -2) {
    const char* e = getenv("T2W_GEMM_PAIR");
    v = (e && e[0] == '0') ? 0 : (e && e[0] == '1') ? 1 : -1;
  }
  if (v >= 0) return v == 1;
  const long long pair_tiles = (long long)((a.M + 255) / 256) * (a.N / 256);
  return a.K * a.taps >= 1536 && pair_tiles >= 3ll * (num_sms() / 2);
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
// faster than the SM delivers them beside the TMA writes; 128 x 256 runs the tensor core at its rate), 128 when N is
// not a multiple of 256 or when 256-column tiles would fill at most half the SMs.  T2W_GEMM_BN=128 / =256 overrides
// the rule for multiples of 256.
int gemm_block_n_for(int N, int M, int epi) {
  (void)epi;
  static int force = -2;
  if (force == -2) {
    const char* e = getenv("T2W_GEMM_BN");
    force = (e && atoi(e) == 128) ? 128 : (e && atoi(e) == 256) ? 256 : 0;
  }
  if (N == 80) return 80;
  if (N % 256 == 0) {
    if (force) return force;
    // With few 128-row blocks the 128 x 256 tiles leave most SMs idle; 128-column tiles double the CTAs at the cost
    // of the tensor core's rate on each (their operands arrive from shared memory more slowly per FLOP).
    const long long tiles = (long long)((M + kBM - 1) / kBM) * (N / 256);
    return 2 * tiles <= num_sms() ? 128 : 256;
  }
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
  if (a.epi == T2W_EPI_RESID && (!a.gate || (reinterpret_cast<uintptr_t>(a.out) & 15) ||
                                 (reinterpret_cast<uintptr_t>(a.gate) & 15) || (reinterpret_cast<uintptr_t>(a.bias) & 15)))
    return T2W_ERR_INVALID;
  if (bn == 80) {
    if (a.epi == T2W_EPI_F32) return launch_impl<80, T2W_EPI_F32, false>(a, st, tmA, tmW, tmC);
    if (a.epi == T2W_EPI_BF16) return launch_impl<80, T2W_EPI_BF16, false>(a, st, tmA, tmW, tmC);
    return T2W_ERR_INVALID;
  }
  if (bn == 256 && use_pair(a)) {
    switch (a.epi) {
      case T2W_EPI_F32: return launch_pair_impl<T2W_EPI_F32>(a, st, tmA, tmW, tmC);
      case T2W_EPI_BF16: return launch_pair_impl<T2W_EPI_BF16>(a, st, tmA, tmW, tmC);
      case T2W_EPI_GELU: return launch_pair_impl<T2W_EPI_GELU>(a, st, tmA, tmW, tmC);
      case T2W_EPI_SILU: return launch_pair_impl<T2W_EPI_SILU>(a, st, tmA, tmW, tmC);
      case T2W_EPI_LEAKY: return launch_pair_impl<T2W_EPI_LEAKY>(a, st, tmA, tmW, tmC);
      case T2W_EPI_QKV: return launch_pair_impl<T2W_EPI_QKV>(a, st, tmA, tmW, tmC);
      case T2W_EPI_RESID: return launch_pair_impl<T2W_EPI_RESID>(a, st, tmA, tmW, tmC);
      default: return T2W_ERR_INVALID;
    }
  }
  if (bn == 256) {
    switch (a.epi) {
      case T2W_EPI_F32: return launch_impl<256, T2W_EPI_F32, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_BF16: return launch_impl<256, T2W_EPI_BF16, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_GELU: return launch_impl<256, T2W_EPI_GELU, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_SILU: return launch_impl<256, T2W_EPI_SILU, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_LEAKY: return launch_impl<256, T2W_EPI_LEAKY, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_QKV: return launch_impl<256, T2W_EPI_QKV, true>(a, st, tmA, tmW, tmC);
      case T2W_EPI_RESID: return launch_impl<256, T2W_EPI_RESID, true>(a, st, tmA, tmW, tmC);
      default: return T2W_ERR_INVALID;
    }
  }
  switch (a.epi) {
    case T2W_EPI_F32: return launch_impl<128, T2W_EPI_F32, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_BF16: return launch_impl<128, T2W_EPI_BF16, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_GELU: return launch_impl<128, T2W_EPI_GELU, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_SILU: return launch_impl<128, T2W_EPI_SILU, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_LEAKY: return launch_impl<128, T2W_EPI_LEAKY, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_QKV: return launch_impl<128, T2W_EPI_QKV, true>(a, st, tmA, tmW, tmC);
    case T2W_EPI_RESID: return launch_impl<128, T2W_EPI_RESID, true>(a, st, tmA, tmW, tmC);
    default: return T2W_ERR_INVALID;
  }
}

}  // namespace t2w
