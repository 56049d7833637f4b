// TF32 tcgen05 implicit-GEMM convolution for the HiFT vocoder: out[m, n] = sum_tap sum_c A[m + tap_row0 + tap * dil, c]
// W[n, tap * Cp + c].
//
// A is the time-major fp32 activation [rows, Cin] with zero rows around every window's data (the "same" padding), W
// the fp32 weight [Cout, taps * Cp]; the tensor core reads both as TF32 (kind::tf32, K = 8 per instruction, fp32
// accumulation in TMEM) — the reference's own reduced-precision option for the upsampling stages (decode_tf32,
// engine/models/token2wav.py:145-210).  Where fp32 is wanted (the f0 predictor and conv_post in every tensor-core mode,
// every convolution in the fp32 tensor-core mode) the same kernel runs in split form (3xTF32): the operands arrive as
// hi + lo pairs of TF32-exact values (hi the value rounded to TF32, lo the remainder rounded to TF32) and the K loop
// runs hi W_hi + hi W_lo + lo W_hi, which leaves the lo x lo term and the pairs' own rounding, about 3 x 2^-24 relative
// per product: fp32-level accuracy on the tensor core.
//
// One persistent CTA per SM, warp-specialised: warp 0 the TMA producer, warp 1 the TMEM allocator and single-thread MMA
// issuer, warps 2-17 the epilogue (TMEM lane quarter w % 4, every fourth 16-column chunk: four warps per quarter, since
// with two the epilogue's instruction latency, not the MMAs, set the pace of the 1-7-tap convolutions), the
// accumulator double-buffered in TMEM so a tile's epilogue overlaps the next tile's MMAs.  Main loop, in one of two
// forms: tap reuse (the usual one) — one A box per 32-channel block covers every tap's rows and each tap's MMAs read it
// from a row offset, W streaming per (tap, block) through its own ring, with tiles of two 128-row halves sharing each W
// box where the halo fits (8 MMAs a step), and the split form's hi / lo boxes where it is used; or one 128 x 32 A box
// and one BN x 32 W box per (tap, segment, block), 128-byte swizzle throughout.  Each epilogue thread owns one output
// row (the TMEM lane it reads) and stores its 16-column chunk directly; a residual update first TMA-loads the warp's
// 32 x 16 block of the residual (out itself, or another buffer of the same layout) into a swizzled shared-memory box
// (issued before the accumulator is ready) and reads its row from there, instead of 32 scattered row reads per warp.
// (Staging the outputs through the box, as TMA stores or as 64-byte row segments, measured slower overall.)
// Output rows: row_mul * m + row_add (a transposed convolution's output phase writes every row_mul-th row of the next
// rate's layout, a tensor map whose row pitch is row_mul rows); rows flagged in `pad` are window padding and stay zero.
// Epilogues: bias (optionally with Snake(out) into a second buffer); Snake(bias + acc) (the ResBlocks' conv1); x +=
// bias + acc with Snake(x_new) into a second buffer (conv2's residual and the next conv1's input; x read from out itself
// or, out of place, from another buffer); ELU (the f0 predictor); leaky ReLU (conv_pre); outputs and second outputs
// optionally as hi / lo pairs for a split-form consumer.  No TMA multicast.
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "tconv.h"

namespace t2w {

namespace {

constexpr int kTBM = 128;
constexpr int kTBK = 32;  // fp32 elements per 128-byte swizzle row
constexpr int kTMaxSmem = 232448;
constexpr int kEpiWarps = 16;         // four per TMEM lane quarter
constexpr int kEC = 16;               // columns per epilogue chunk
constexpr int kEBox = 32 * kEC * 4;   // one epilogue warp's 32 x 16 fp32 residual box (64-byte rows, 64-byte swizzle)
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct TCfg {
  static constexpr int A_BYTES = kTBM * kTBK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * kTBK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_BYTES = kEpiWarps * kEBox;
  static constexpr int FIXED = 1024 + 512;
  static constexpr int STAGES_FIT = (kTMaxSmem - FIXED - EPI_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int TMEM_COLS = (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + FIXED;
  static_assert(STAGES >= 3, "stages");
  static_assert(SMEM <= kTMaxSmem, "shared memory");
};

// Tap-reuse form (128 + (taps - 1) dil <= 256): one A box per 32-channel block covers every tap's rows
// (128 + (taps - 1) dil of them) and each tap's MMAs read it from a row offset; W streams per (tap, block) through its
// own ring.  A traffic per tile drops from taps x 128 rows to 128 + (taps - 1) dil rows per channel block.  The
// operand descriptor of a tap simply starts tap x dil 128-byte rows into the box, with the matrix base offset field
// left 0: the 128-byte swizzle the TMA wrote is a function of the absolute shared-memory address bits, and the MMA
// reads it back from any row start (measured: every offset 1-12 rows exact; setting the field to the start's row
// phase breaks every offset that is not a multiple of 8).
//
// MH = 2 (BN <= 128): a CTA tile is two 128-row halves that share every W box, each half its own TMEM accumulator: a
// (tap, block) step issues 8 MMAs instead of 4.  Each step of the pipeline costs ~220 ns beyond its MMAs (measured:
// doubling a step's MMAs added 100 ns to its 325), so twice the MMA work per step pays that once per 256 rows.
//
// SPLIT (split form, MH = 1): a channel block's A boxes are its hi and lo parts, a step's W boxes W_hi and W_lo, and a
// step issues hi W_hi, hi W_lo and lo W_hi (12 MMAs).
constexpr int kUASlots = 2;
template <int MH, bool SPLIT = false>
constexpr int ua_rows() { return (MH == 2 || SPLIT) ? 192 : 256; }  // A box capacity: 128 + (taps - 1) dil rows at most
template <int BN, int MH, bool SPLIT = false>
struct TCfgU {
  static constexpr int B_BYTES = BN * kTBK * 4;
  static constexpr int NA = SPLIT ? 2 : 1;                     // A boxes per half and channel block (hi, lo)
  static constexpr int NW = SPLIT ? 2 : 1;                     // W boxes per step (W_hi, W_lo)
  static constexpr int ABOX = ua_rows<MH, SPLIT>() * kTBK * 4;  // one A box
  static constexpr int ASLOT = MH * NA * ABOX;                 // a channel block's A boxes
  static constexpr int WSTEP = NW * B_BYTES;
  static constexpr int WFIT = (kTMaxSmem - TCfg<BN>::FIXED - TCfg<BN>::EPI_BYTES - kUASlots * ASLOT) / WSTEP;
  static constexpr int WSTAGES = WFIT > 8 ? 8 : WFIT;
  static constexpr int SMEM = kUASlots * ASLOT + WSTAGES * WSTEP + TCfg<BN>::EPI_BYTES + TCfg<BN>::FIXED;
  static constexpr int TMEM_COLS = (2 * MH * BN <= 128) ? 128 : (2 * MH * BN <= 256) ? 256 : 512;
  static_assert(2 * MH * BN <= 512, "TMEM");
  static_assert(WSTAGES >= 3, "stages");
  static_assert(SMEM <= kTMaxSmem, "shared memory");
};

struct TDev {
  int M, N, Cin, taps, tap_row0, dil, tiles_n, num_tiles;
  int split_in, split_out, split_out2;
  float slope;  // TCONV_LEAKY
  long long ldo2;
  int urows;  // tap-reuse form: rows of the A box (0: one 128-row A box per tap)
  const float* bias;
  float* out;
  float* out2;
  int resid_oop;  // the residual is read from another buffer than out
  const uint8_t* pad;
  long long ldo;  // floats between consecutive output rows of the layout (row_mul * m + row_add indexes them)
  int row_mul, row_add;
  int epi;
  const float* alpha;
  const float* inv;
  int has_out2;
  int* err;
};

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  // D fp32 (bits 4-5 = 1), A and B TF32 (format 2 at bits 7-9 and 10-12), both K-major, N >> 3, M >> 4
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

T2W_DEV void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// sin for the Snake activation on this TF32 path: the argument reduced to [-pi, pi] with 2 pi split into two floats
// (Cody-Waite: n = rint(x / 2 pi), r = (x - n hi) - n lo, the products exact enough for |n| < 2^12), then the
// hardware approximation __sinf, whose absolute error there is about 2^-21.  That is ~1e-6 on a Snake output, three
// orders below the TF32 operand rounding of the convolutions around it.
__device__ __forceinline__ float sin_reduced(float x) {
  const float n = rintf(x * 0.159154943091895336f);
  float r = fmaf(-n, 6.28318548202514648f, x);
  r = fmaf(-n, -1.74845553146951715e-07f, r);
  return __sinf(r);
}
__device__ __forceinline__ float snake_f(float x, float a, float inv) {
  const float s = sin_reduced(x * a);
  return x + inv * (s * s);
}

// 16-byte chunk `c` (0-3) of row `r` of a 64-byte-row box staged with the 64-byte swizzle (chunk index XOR bits 7-8
// of the row's byte offset, (r / 2) % 4).
__device__ __forceinline__ float4* box_chunk(uint8_t* box, int r, int c) {
  return reinterpret_cast<float4*>(box + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}
// fp32 rounded to the nearest TF32 value (half of the dropped unit added to the bit pattern, then the 13 low mantissa
// bits cleared): a split x = hi + lo with hi = tf32_rn(x), lo = tf32_rn(x - hi) leaves |x - hi - lo| <= 2^-24 |x|.
__device__ __forceinline__ float tf32_rn(float x) { return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u); }
// Four outputs j of a row chunk: plain, or as the split form's [hi | lo] pair (the lo part n columns to the right).
__device__ __forceinline__ void store4(float* row, int j, float4 y, bool split, int n) {
  if (split) {
    const float4 hi = make_float4(tf32_rn(y.x), tf32_rn(y.y), tf32_rn(y.z), tf32_rn(y.w));
    reinterpret_cast<float4*>(row + n)[j] =
        make_float4(tf32_rn(y.x - hi.x), tf32_rn(y.y - hi.y), tf32_rn(y.z - hi.z), tf32_rn(y.w - hi.w));
    y = hi;
  }
  reinterpret_cast<float4*>(row)[j] = y;
}

template <int BN, bool UNION, int MH, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_tconv(const __grid_constant__ CUtensorMap tmA,
                                                  const __grid_constant__ CUtensorMap tmW,
                                                  const __grid_constant__ CUtensorMap tmR, const TDev p) {
  static_assert(MH == 1 || UNION, "two-half tiles in the tap-reuse form only");
  static_assert(!SPLIT || (UNION && MH == 1), "split form in the tap-reuse path: one half per tile");
  using C = TCfg<BN>;
  using CU = TCfgU<BN, MH, SPLIT>;
  constexpr int WSTEP = UNION ? CU::WSTEP : C::B_BYTES;
  constexpr int TM = kTBM * MH;                                // rows per CTA tile
  constexpr int NST = UNION ? CU::WSTAGES : C::STAGES;        // W (and, in the per-tap form, A) ring depth
  constexpr int A_RING = UNION ? kUASlots * CU::ASLOT : C::STAGES * C::A_BYTES;
  constexpr int TMEM_COLS = UNION ? CU::TMEM_COLS : C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + A_RING;
  uint8_t* sE = sB + NST * WSTEP;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + C::EPI_BYTES);
  uint64_t* empty = full + NST;
  uint64_t* tfull = empty + NST;
  uint64_t* tempty = tfull + 2;
  uint64_t* ebar = tempty + 2;
  uint64_t* afull = ebar + kEpiWarps;  // tap-reuse form: the A slots
  uint64_t* aempty = afull + kUASlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + kUASlots);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kUASlots; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&ebar[w], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmR);
  }
  pdl_wait();
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch();
  const uint32_t tmem = *tmem_slot;
  const int kb_per_seg = (p.Cin + kTBK - 1) / kTBK;  // channels past Cin in the last block read as zero
  const int cpad = kb_per_seg * kTBK;                  // W's columns per (tap, segment)
  const int segs = p.split_in ? 3 : 1;
  const int kb_per_tap = kb_per_seg * segs;
  const int num_kb = kb_per_tap * p.taps;

  if (UNION && warp == 0) {
    if (lane == 0) {
      int stage = 0, as = 0;
      uint32_t phase = 0, aph = 0;
      bool ok = true;
      const uint32_t abytes = (uint32_t)p.urows * kTBK * 4;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * TM, n0 = (tile % p.tiles_n) * BN;
        for (int cb = 0; cb < kb_per_seg && ok; ++cb) {
          if (!(ok = mbar_wait(&aempty[as], aph ^ 1u, p.err))) break;
          mbar_expect_tx(&afull[as], MH * CU::NA * abytes);
#pragma unroll
          for (int h = 0; h < MH; ++h)
#pragma unroll
            for (int sa = 0; sa < CU::NA; ++sa)  // split form: hi at channel cb, lo Cin channels on
              tma_load_2d(sA + as * CU::ASLOT + (h * CU::NA + sa) * CU::ABOX, &tmA, sa * p.Cin + cb * kTBK,
                          m0 + h * kTBM + p.tap_row0, &afull[as]);
          if (++as == kUASlots) {
            as = 0;
            aph ^= 1u;
          }
          for (int tap = 0; tap < p.taps; ++tap) {
            if (!(ok = mbar_wait(&empty[stage], phase ^ 1u, p.err))) break;
            mbar_expect_tx(&full[stage], CU::WSTEP);
#pragma unroll
            for (int sw = 0; sw < CU::NW; ++sw)  // split form: W_hi, W_lo of the tap's [W_hi | W_lo | W_hi]
              tma_load_2d(sB + stage * CU::WSTEP + sw * C::B_BYTES, &tmW, (tap * segs + sw) * cpad + cb * kTBK, n0,
                          &full[stage]);
            if (++stage == NST) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    }
  } else if (UNION && warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kTBM, BN);
      int stage = 0, as = 0;
      uint32_t phase = 0, aph = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!(ok = mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1u, p.err))) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * MH * BN;
        for (int cb = 0; cb < kb_per_seg && ok; ++cb) {
          if (!(ok = mbar_wait(&afull[as], aph, p.err))) break;
          const uint32_t a_slot = smem_u32(sA + as * CU::ASLOT);
          for (int tap = 0; tap < p.taps; ++tap) {
            if (!(ok = mbar_wait(&full[stage], phase, p.err))) break;
            tc_fence_after();
            const uint32_t b_step = smem_u32(sB + stage * CU::WSTEP);
#pragma unroll
            for (int h = 0; h < MH; ++h) {
#pragma unroll
              for (int pr = 0; pr < (SPLIT ? 3 : 1); ++pr) {  // split form: (hi, W_hi), (hi, W_lo), (lo, W_hi)
                const int sa = pr == 2 ? 1 : 0, sw = pr == 1 ? 1 : 0;
                const uint32_t a0 = a_slot + (h * CU::NA + sa) * CU::ABOX + (uint32_t)(tap * p.dil) * 128u;
                const uint32_t b0 = b_step + sw * C::B_BYTES;
#pragma unroll
                for (int k = 0; k < kTBK / 8; ++k)
                  umma_tf32(d + h * BN, sdesc_sw128(a0 + 32 * k, 1024, 16), sdesc_sw128(b0 + 32 * k, 1024, 16), idesc,
                            (cb | tap | pr | k) != 0 ? 1u : 0u);
              }
            }
            umma_commit(&empty[stage]);
            if (++stage == NST) {
              stage = 0;
              phase ^= 1u;
            }
          }
          umma_commit(&aempty[as]);  // after the block's last MMA (commit tracks every MMA issued before it)
          if (++as == kUASlots) {
            as = 0;
            aph ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * TM, n0 = (tile % p.tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!(ok = mbar_wait(&empty[stage], phase ^ 1u, p.err))) break;
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          // segment 0: hi x W_hi, 1: hi x W_lo, 2: lo x W_hi (split form); the plain form has segment 0 only
          const int tap = kb / kb_per_tap, r = kb - tap * kb_per_tap, seg = r / kb_per_seg;
          const int kk = (r - seg * kb_per_seg) * kTBK;
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, (seg == 2 ? p.Cin : 0) + kk, m0 + p.tap_row0 + tap * p.dil,
                      &full[stage]);
          tma_load_2d(sB + stage * C::B_BYTES, &tmW, (tap * segs + seg) * cpad + kk, n0, &full[stage]);
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kTBM, BN);
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
          for (int k = 0; k < kTBK / 8; ++k)
            umma_tf32(d, sdesc_sw128(a0 + 32 * k, 1024, 16), sdesc_sw128(b0 + 32 * k, 1024, 16), idesc,
                      (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    const int grp = ew >> 2;  // this warp's chunks: grp, grp + 4, ... of the tile's 16-column chunks
    uint8_t* box = sE + ew * kEBox;
    uint64_t* eb = &ebar[ew];
    uint32_t eph = 0;
    const bool resid = p.epi == TCONV_RESID;
    bool pending = false;  // a residual load of this warp in flight
    auto load_resid = [&](int c0, int r0) {
      if (lane == 0) {
        mbar_expect_tx(eb, kEBox);
        tma_load_2d(box, &tmR, c0, r0, eb);
      }
      pending = true;
    };
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const int m0 = (tile / p.tiles_n) * TM, n0 = (tile % p.tiles_n) * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * MH * BN;
      if (resid && grp < BN / kEC) load_resid(n0 + kEC * grp, m0 + q * 32);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], (it >> 1) & 1, p.err))) {
        if (pending) mbar_wait(eb, eph, p.err);
        break;
      }
      tc_fence_after();
      if (grp >= BN / kEC) {  // a 32-column tile: two of the four warp groups have no chunk of their own
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
      bool ok = true;
#pragma unroll 1
      for (int h = 0; h < MH && ok; ++h) {
      const int r0 = m0 + h * kTBM + q * 32;  // this warp's first row of the half
      const long long orow = (long long)p.row_mul * (r0 + lane) + p.row_add;
      const bool live = !p.pad[orow];
#pragma unroll 1
      for (int b = grp; b < BN / kEC; b += 4) {
        const int c0 = n0 + kEC * b;
        float v[kEC];
        tmem_ld16(taddr + h * BN + kEC * b, v);
        if (h == MH - 1 && b + 4 >= BN / kEC) {  // this warp's last load of the accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        float* dst = p.out + orow * p.ldo + c0;
        if (resid) {
          ok = __all_sync(0xffffffffu, mbar_wait(eb, eph, p.err));
          eph ^= 1u;
          pending = false;
          if (!ok) break;
          float4 xb[kEC / 4];  // this row's residual chunk, out of the box before the next load refills it
#pragma unroll
          for (int j = 0; j < kEC / 4; ++j) xb[j] = *box_chunk(box, lane, j);
          fence_proxy_async_smem();  // every lane's reads of the box come before the next load overwrites it
          __syncwarp();
          if (b + 4 < BN / kEC)
            load_resid(c0 + 4 * kEC, r0);  // this half's next chunk
          else if (h + 1 < MH)
            load_resid(n0 + kEC * grp, r0 + kTBM);  // the next half's first chunk
          float* dst2 = p.has_out2 ? p.out2 + orow * p.ldo2 + c0 : nullptr;
          if (!live && p.resid_oop) {  // a padding row of an out-of-place update: the residual's (zero) row
#pragma unroll
            for (int j = 0; j < kEC / 4; ++j) reinterpret_cast<float4*>(dst)[j] = xb[j];
          }
#pragma unroll
          for (int j = 0; j < kEC / 4 && live; ++j) {  // padding rows of an in-place update keep their (zero) values
            const float4 x = xb[j];
            const float4 bb = __ldg(reinterpret_cast<const float4*>(p.bias + c0) + j);
            const float4 y = make_float4(x.x + (v[4 * j] + bb.x), x.y + (v[4 * j + 1] + bb.y),
                                         x.z + (v[4 * j + 2] + bb.z), x.w + (v[4 * j + 3] + bb.w));
            reinterpret_cast<float4*>(dst)[j] = y;
            if (dst2) {
              const float4 a = __ldg(reinterpret_cast<const float4*>(p.alpha + c0) + j);
              const float4 iv = __ldg(reinterpret_cast<const float4*>(p.inv + c0) + j);
              store4(dst2, j,
                     make_float4(snake_f(y.x, a.x, iv.x), snake_f(y.y, a.y, iv.y), snake_f(y.z, a.z, iv.z),
                                 snake_f(y.w, a.w, iv.w)),
                     p.split_out2, p.N);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kEC / 4; ++j) {
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f), z = y;
            if (live) {
              const float4 bb = __ldg(reinterpret_cast<const float4*>(p.bias + c0) + j);
              y = make_float4(v[4 * j] + bb.x, v[4 * j + 1] + bb.y, v[4 * j + 2] + bb.z, v[4 * j + 3] + bb.w);
              if (p.has_out2) {  // bias epilogue: the next ResBlock's first Snake of the output beside it
                const float4 a = __ldg(reinterpret_cast<const float4*>(p.alpha + c0) + j);
                const float4 iv = __ldg(reinterpret_cast<const float4*>(p.inv + c0) + j);
                z = make_float4(snake_f(y.x, a.x, iv.x), snake_f(y.y, a.y, iv.y), snake_f(y.z, a.z, iv.z),
                                snake_f(y.w, a.w, iv.w));
              }
              if (p.epi == TCONV_SNAKE) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(p.alpha + c0) + j);
                const float4 iv = __ldg(reinterpret_cast<const float4*>(p.inv + c0) + j);
                y = make_float4(snake_f(y.x, a.x, iv.x), snake_f(y.y, a.y, iv.y), snake_f(y.z, a.z, iv.z),
                                snake_f(y.w, a.w, iv.w));
              } else if (p.epi == TCONV_ELU) {
                y = make_float4(y.x > 0.f ? y.x : expm1f(y.x), y.y > 0.f ? y.y : expm1f(y.y),
                                y.z > 0.f ? y.z : expm1f(y.z), y.w > 0.f ? y.w : expm1f(y.w));
              } else if (p.epi == TCONV_LEAKY) {
                y = make_float4(y.x > 0.f ? y.x : y.x * p.slope, y.y > 0.f ? y.y : y.y * p.slope,
                                y.z > 0.f ? y.z : y.z * p.slope, y.w > 0.f ? y.w : y.w * p.slope);
              }
            }
            store4(dst, j, y, p.split_out, p.N);
            if (p.has_out2) store4(p.out2 + orow * p.ldo2 + c0, j, z, p.split_out2, p.N);
          }
        }
      }
      }
      if (!ok) break;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int BN, bool UNION, int MH, bool SPLIT = false>
int launch_impl(const TConvArgs& a, cudaStream_t st) {
  constexpr int SMEM = UNION ? TCfgU<BN, MH, SPLIT>::SMEM : TCfg<BN>::SMEM;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = smem_attr_once(k_tconv<BN, UNION, MH, SPLIT>, SMEM, attr_done);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  const int segs = a.split_in ? 3 : 1;
  const uint64_t out_cols = (uint64_t)a.N * (a.split_out ? 2 : 1);
  const uint64_t out_pitch = (uint64_t)a.row_mul * a.ldo * 4;
  CUtensorMap ma, mw, mr;
  const uint64_t cpad = (uint64_t)(a.Cin + kTBK - 1) / kTBK * kTBK;
  const int urows = UNION ? ((a.taps - 1) * a.dil + kTBM + 7) / 8 * 8 : 0;  // every tap's rows of a 128-row tile
  if (!make_tmap_2d(&ma, a.A, 4, (uint64_t)a.rows_a, (uint64_t)a.Cin * (a.split_in ? 2 : 1), (uint64_t)a.lda * 4,
                    UNION ? urows : kTBM, kTBK) ||
      !make_tmap_2d(&mw, a.W, 4, (uint64_t)a.N, cpad * a.taps * segs, cpad * a.taps * segs * 4, BN, kTBK) ||
      !make_tmap_2d_ex(&mr, (a.resid_in ? a.resid_in : a.out) + (long long)a.row_add * a.ldo, 4, (uint64_t)a.M,
                       out_cols, out_pitch, 32, kEC, kEC * 4))
    return T2W_ERR_INVALID;
  TDev p;
  p.M = a.M;
  p.N = a.N;
  p.Cin = a.Cin;
  p.taps = a.taps;
  p.tap_row0 = a.tap_row0;
  p.dil = a.dil;
  p.tiles_n = a.N / BN;
  p.num_tiles = (a.M / (kTBM * MH)) * p.tiles_n;
  p.split_in = a.split_in;
  p.split_out = a.split_out;
  p.split_out2 = a.split_out2;
  p.slope = a.slope;
  p.ldo2 = a.ldo2 ? a.ldo2 : a.ldo;
  p.urows = urows;
  p.bias = a.bias;
  p.out = a.out;
  p.out2 = a.out2;
  p.resid_oop = a.resid_in != nullptr && a.resid_in != a.out;
  p.pad = a.pad;
  p.ldo = a.ldo;
  p.row_mul = a.row_mul;
  p.row_add = a.row_add;
  p.epi = a.epi;
  p.alpha = a.alpha;
  p.inv = a.inv;
  p.has_out2 = a.out2 != nullptr;
  p.err = a.err;
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  e = launch_k(k_tconv<BN, UNION, MH, SPLIT>, dim3(grid), dim3(kThreads), SMEM, st, ma, mw, mr, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace

int launch_tconv(const TConvArgs& a, cudaStream_t st) {
  if (!a.A || !a.W || !a.bias || !a.out || !a.pad || a.M <= 0 || a.M % kTBM || a.Cin <= 0 || a.Cin % 4 ||
      (a.split_in && a.Cin % kTBK) ||
      a.taps < 1 || a.rows_a <= 0 || a.lda < a.Cin * (a.split_in ? 2 : 1) || a.lda % 4 || a.ldo % 4 ||
      a.ldo < (long long)a.N * (a.split_out ? 2 : 1) || a.row_mul < 1 || a.row_add < 0 || a.row_add >= a.row_mul ||
      a.epi < TCONV_BIAS || a.epi > TCONV_LEAKY || (a.epi == TCONV_SNAKE && (!a.alpha || !a.inv)) ||
      (a.out2 && ((a.epi != TCONV_RESID && a.epi != TCONV_BIAS) || !a.alpha || !a.inv)) ||
      (a.split_out && a.epi == TCONV_RESID) || (a.split_out2 && !a.out2) || a.ldo2 % 4 ||
      (a.out2 && (a.ldo2 ? a.ldo2 : a.ldo) < (long long)a.N * (a.split_out2 ? 2 : 1)) ||
      (reinterpret_cast<uintptr_t>(a.out) & 15) || (a.out2 && (reinterpret_cast<uintptr_t>(a.out2) & 15)) ||
      (a.resid_in && (a.epi != TCONV_RESID || (reinterpret_cast<uintptr_t>(a.resid_in) & 15))) ||
      (reinterpret_cast<uintptr_t>(a.bias) & 15))
    return T2W_ERR_INVALID;
  // the tap-reuse form when every tap's rows fit one A box; with two 128-row halves per tile when they fit the smaller
  // boxes of that form and M is a multiple of 256 (tiles of up to 128 columns)
  const long long ext = (long long)(a.taps - 1) * a.dil + kTBM;
  const bool u = !a.split_in && ext <= ua_rows<1>();
  const bool u2 = u && ext <= ua_rows<2>() && a.M % (2 * kTBM) == 0;
  if (a.split_in && ext <= ua_rows<1, true>()) {  // the split form's tap-reuse path (tiles of up to 128 columns)
    if (a.N % 128 == 0) return launch_impl<128, true, 1, true>(a, st);
    if (a.N == 64) return launch_impl<64, true, 1, true>(a, st);
    if (a.N == 32) return launch_impl<32, true, 1, true>(a, st);
  }
  if (a.N % 128 == 0 && a.N >= 256 && (long long)(a.M / kTBM) * (a.N / 256) >= num_sms())
    return u ? launch_impl<256, true, 1>(a, st) : launch_impl<256, false, 1>(a, st);
  if (a.N % 128 == 0)
    return u2 ? launch_impl<128, true, 2>(a, st) : u ? launch_impl<128, true, 1>(a, st) : launch_impl<128, false, 1>(a, st);
  if (a.N == 64)
    return u2 ? launch_impl<64, true, 2>(a, st) : u ? launch_impl<64, true, 1>(a, st) : launch_impl<64, false, 1>(a, st);
  if (a.N == 32)
    return u2 ? launch_impl<32, true, 2>(a, st) : u ? launch_impl<32, true, 1>(a, st) : launch_impl<32, false, 1>(a, st);
  return T2W_ERR_INVALID;
}

}  // namespace t2w
