// Flow-encoder kernels: relative-position attention on tcgen05 tensor cores, and the encoder's row, cache and gather
// kernels.  The GEMMs of the encoder (input / up embeddings, the convolutions as implicit-im2col taps, QKV, the
// attention output, the swish feed-forward, encoder_proj) run on k_gemm (gemm.cu).
//
// Relative-position attention (the conformer layers' RelPositionMultiHeadedAttention; the reference runs it through
// its third-party module, driven by engine/runtime/token2wav_batch.py:42-79).  For query i (at position K - T + i of a
// sequence of K keys whose last T are the window's own) and key j:
//   score(i, j) = [(q_i + u) . k_j + (q_i + v) . P(r)] / sqrt(64),   r = (K - T + i) - j,
// P(r) = linear_pos(pe(r)) per head, read from a table indexed by r (the ESPnet rel_shift of a [T, 2K - 1] product
// puts exactly P(r) at (i, j)).  One CTA per (128-query tile, head); keys in tiles of 32.  Per tile:
//   S  = (Q + u) K^T              (M 128, N 32, K 64)  into TMEM columns [0, 32)
//   B  = (Q + v) Pband^T          (M 128, N 160, K 64) into TMEM columns [32, 192), Pband = P(rb) .. P(rb + 159),
//        rb = K - T + q_pos - j0 - 31: query row p and tile key k need band column 31 + p - k
//   the softmax thread of row p loads S and the 64 band columns of its warp (32 w .. 32 w + 63), shifts the band by its
//   lane with five predicated stages (band column 31 + p - k sits at register 31 - k after the shift), adds, and keeps
//   a running max that it raises only when a tile's max exceeds it by more than 8 (then O is rescaled in TMEM);
//   P = 2^(s c - m) is written back over S as bf16 pairs and O += P V (M 128, N 64, K 32; V MN-major) accumulates in
//   TMEM columns [192, 256).
// Warps: 0 = producer (TMA of the Q tiles and of each tile's band of the position table; the warp gathers K / V rows
// from the key pool with 16-byte cp.async into the 128-byte-swizzled layout a TMA tile has), 1 = TMEM allocator and
// single-thread MMA issuer, 2-5 = softmax (one query row per thread = TMEM lane).  256 TMEM columns and 90 KB of shared
// memory per CTA, so two CTAs share an SM and one's softmax overlaps the other's MMAs.  No TMA multicast.
#include <atomic>

#include "common.cuh"
#include "enc_kernels.h"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kRQ = 128;              // queries per CTA
constexpr int kRK = 32;               // keys per tile
constexpr int kRBand = kRQ + kRK;     // band rows per tile at most (159 used)
constexpr int kRBox = 32;             // rows of one position-table TMA box
constexpr int kD = 64;
constexpr int kQBytes = kRQ * kD * 2;        // 16 KB per Q tile (q + u, q + v)
constexpr int kKBytes = kRK * kD * 2;        // 4 KB for K, 4 KB for V
constexpr int kPBytes = kRBand * kD * 2;     // 20 KB of position rows at most
constexpr int kKVStages = 4;                 // K / V gathers from the pool (HBM): four tiles in flight
constexpr int kBStages = 2;                  // position bands (L2-resident table), freed as soon as S is computed
constexpr int kKVOff = 2 * kQBytes;
constexpr int kBOff = kKVOff + kKVStages * 2 * kKBytes;
constexpr int kBarOff = kBOff + kBStages * kPBytes;  // 104 KB
constexpr int kRSmem = 1024 + kBarOff + 256;
constexpr int kRTmem = 256;  // S / P at [0, 32), band at [32, 32 + band rows), O at [192, 256)
constexpr int kRThreads = 224;
constexpr float kRescale = 8.f;

struct RelBars {
  uint64_t q_full, kv_full[kKVStages], kv_empty[kKVStages], b_full[kBStages], b_empty[kBStages], s_full, p_full, o_done;
};

T2W_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
T2W_DEV void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// O (+)= P V with P from TMEM (A operand: 2 bf16 keys per 32-bit column) and V from shared memory.
T2W_DEV void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
T2W_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
T2W_DEV void tmem_st32f(uint32_t taddr, const float (&f)[32]) {
  uint32_t v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(f[i]);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
T2W_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 lanes x 32 columns without waiting: the caller issues tmem_ld_wait() before it reads the registers.
T2W_DEV void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Band rows an item needs: its active query rows (up to 128 from q_pos) in whole warps, plus the tile's 32 keys.
T2W_DEV int band_rows(const RelWork& w) {
  const int ar = min(kRQ, w.T - w.q_pos);
  return kRBox * ((ar + 31) / 32) + kRK;
}

__global__ void __launch_bounds__(kRThreads, 2) k_relattn(const __grid_constant__ CUtensorMap tm_q,
                                                          const __grid_constant__ CUtensorMap tm_pos, const RelArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qu = smem;
  uint8_t* qv = smem + kQBytes;
  RelBars* bars = reinterpret_cast<RelBars*>(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.heads * kD;
  const int h = blockIdx.x % p.heads;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&bars->kv_full[s], 32);  // one cp.async arrival per gathering lane
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&bars->b_full[s], 1);
      mbar_init(&bars->b_empty[s], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->p_full, 4);
    mbar_init(&bars->o_done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_pos);
  }
  pdl_wait();
  const RelWork w = p.work[blockIdx.x / p.heads];
  const int n_kt = (w.K + kRK - 1) / kRK;
  const int nb = band_rows(w);
  if (warp == 1) {
    tmem_alloc(tmem_slot, kRTmem);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // K / V gathers: the whole warp copies each 32-key tile from the pool with 16-byte cp.async into the 128-byte
    // swizzled layout a TMA tile has (chunk c of row r at chunk c ^ (r % 8)); keys past K are zero-filled.  The slot
    // of the next tile's key is loaded while this tile's copies are issued.
    const __nv_bfloat16* kcol = p.pool + h * kD;
    const __nv_bfloat16* vcol = p.pool + H + h * kD;
    auto slot_of = [&](int key) { return key < w.K ? __ldg(p.kv_idx + w.kv_off + key) : 0; };
    int nxt = slot_of(lane);
    bool ok = true;
    for (int t = 0; t < n_kt && ok; ++t) {
      const int st = t % kKVStages;
      const int cur = nxt;
      if (t + 1 < n_kt) nxt = slot_of((t + 1) * kRK + lane);
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&bars->kv_empty[st], ((t / kKVStages) & 1) ^ 1u, p.err)))) break;
      const uint32_t ks = smem_u32(smem + kKVOff + st * 2 * kKBytes), vs = ks + kKBytes;
      // eight consecutive lanes copy one key row's eight 16-byte chunks (four whole 128-byte rows per copy
      // instruction); row R's slot comes from lane R, which loaded it
      const int c = lane & 7;
#pragma unroll
      for (int i = 0; i < kRK / 4; ++i) {
        const int R = 4 * i + (lane >> 3);
        const size_t slot = (size_t)__shfl_sync(0xffffffffu, cur, R);
        const uint32_t nbytes = (t * kRK + R < w.K) ? 16u : 0u;
        const uint32_t off = R * 128 + ((c ^ (R & 7)) << 4);
        cp_async16(ks + off, kcol + slot * p.pool_ld + 8 * c, nbytes);
        cp_async16(vs + off, vcol + slot * p.pool_ld + 8 * c, nbytes);
      }
      cp_async_arrive_noinc(&bars->kv_full[st]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy of this warp lands after the CTA has moved on
  } else if (warp == 6) {
    if (lane == 0) {  // TMA: the Q tiles, then each tile's band of the position table in 32-row boxes
      mbar_expect_tx(&bars->q_full, 2 * kQBytes);
      tma_load_2d(qu, &tm_q, h * kD, w.q_row, &bars->q_full);
      tma_load_2d(qv, &tm_q, H + h * kD, w.q_row, &bars->q_full);
      for (int t = 0; t < n_kt; ++t) {
        const int st = t % kBStages;
        if (!mbar_wait(&bars->b_empty[st], ((t / kBStages) & 1) ^ 1u, p.err)) break;
        uint8_t* band = smem + kBOff + st * kPBytes;
        const int rb = w.K - w.T + w.q_pos - t * kRK - (kRK - 1) + p.r0;
        mbar_expect_tx(&bars->b_full[st], nb * kD * 2);
        for (int i = 0; i < nb / kRBox; ++i)
          tma_load_2d(band + i * kRBox * kD * 2, &tm_pos, h * kD, rb + i * kRBox, &bars->b_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(kRQ, kRK);
      const uint32_t idesc_b = idesc_bf16(kRQ, nb);
      constexpr uint32_t idesc_pv = idesc_bf16(kRQ, kD, /*b_mn_major=*/true);
      bool ok = mbar_wait(&bars->q_full, 0, p.err);
      const uint32_t q0 = smem_u32(qu), q1 = smem_u32(qv);
      for (int t = 0; t < n_kt && ok; ++t) {
        const int st = t % kKVStages, sb = t % kBStages;
        if (!(ok = mbar_wait(&bars->kv_full[st], (t / kKVStages) & 1, p.err))) break;
        if (!(ok = mbar_wait(&bars->b_full[sb], (t / kBStages) & 1, p.err))) break;
        fence_proxy_async_smem();  // the K / V rows were written by cp.async through the generic proxy
        tc_fence_after();
        const uint32_t ks = smem_u32(smem + kKVOff + st * 2 * kKBytes), vs = ks + kKBytes;
        const uint32_t ps = smem_u32(smem + kBOff + sb * kPBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16(tmem, sdesc_sw128(q0 + 32 * kk, 1024, 16), sdesc_sw128(ks + 32 * kk, 1024, 16), idesc_s, kk ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16(tmem + 32, sdesc_sw128(q1 + 32 * kk, 1024, 16), sdesc_sw128(ps + 32 * kk, 1024, 16), idesc_b,
                   kk ? 1u : 0u);
        umma_commit(&bars->s_full);
        umma_commit(&bars->b_empty[sb]);
        if (!(ok = mbar_wait(&bars->p_full, t & 1, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kRK / 16; ++kk)
          umma_ts(tmem + 192, tmem + 8 * kk, sdesc_sw128(vs + kk * 16 * 128, 1024, 8192), idesc_pv,
                  (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars->kv_empty[st]);
      }
      umma_commit(&bars->o_done);
    }
  } else {
    const int qw = warp & 3;  // TMEM lane quarter
    const int row = qw * 32 + lane;
    const int qi = w.q_pos + row;
    const bool active = qi < w.T;
    const bool idle = __all_sync(0xffffffffu, !active);
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < n_kt; ++t) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full, t & 1, p.err)))) break;
      tc_fence_after();
      if (!idle) {
        uint32_t sr[32], b[64];
        float s[32];
        // the scores and the warp's 64 band columns, three loads in flight and one wait
        tmem_ld32_nowait(tmem + lanes, sr);
        tmem_ld32_nowait(tmem + lanes + 32 + 32 * qw, b);
        tmem_ld32_nowait(tmem + lanes + 64 + 32 * qw, b + 32);
        tmem_ld_wait();
        // shift the warp's band by this lane, b[x] <- b[x + lane] for x < 32: five stages of bitwise selects on the
        // lane's bits (one LOP3 per element, no branches)
        {
          const uint32_t m16 = 0u - ((lane >> 4) & 1u), m8 = 0u - ((lane >> 3) & 1u), m4 = 0u - ((lane >> 2) & 1u),
                         m2 = 0u - ((lane >> 1) & 1u), m1 = 0u - (lane & 1u);
#pragma unroll
          for (int x = 0; x < 47; ++x) b[x] = (b[x + 16] & m16) | (b[x] & ~m16);
#pragma unroll
          for (int x = 0; x < 39; ++x) b[x] = (b[x + 8] & m8) | (b[x] & ~m8);
#pragma unroll
          for (int x = 0; x < 35; ++x) b[x] = (b[x + 4] & m4) | (b[x] & ~m4);
#pragma unroll
          for (int x = 0; x < 33; ++x) b[x] = (b[x + 2] & m2) | (b[x] & ~m2);
#pragma unroll
          for (int x = 0; x < 32; ++x) b[x] = (b[x + 1] & m1) | (b[x] & ~m1);
        }
        const int kb = t * kRK;
#pragma unroll
        for (int k = 0; k < kRK; ++k)
          s[k] = (kb + k < w.K) ? __uint_as_float(sr[k]) + __uint_as_float(b[kRK - 1 - k]) : -INFINITY;
        float mq[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          mq[c] = fmax3(s[8 * c], s[8 * c + 1], s[8 * c + 2]);
          mq[c] = fmax3(mq[c], s[8 * c + 3], s[8 * c + 4]);
          mq[c] = fmax3(mq[c], s[8 * c + 5], s[8 * c + 6]);
          mq[c] = fmaxf(mq[c], s[8 * c + 7]);
        }
        float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * p.scale_log2;
        const bool raise = mx > m + kRescale;
        const float m_old = m;
        m = raise ? mx : m;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        uint32_t u[16];
        float rs = 0.f;
#pragma unroll
        for (int k = 0; k < kRK / 2; ++k) {
          const float e0 = exp2_approx(fmaf(s[2 * k], p.scale_log2, -m_use));
          const float e1 = exp2_approx(fmaf(s[2 * k + 1], p.scale_log2, -m_use));
          rs += e0 + e1;
          u[k] = pack_bf16x2(e0, e1);
        }
        const float f = raise ? exp2_approx(m_old - m) : 1.f;  // 2^-inf = 0 on the first tile
        l = l * f + rs;
        tmem_st16(tmem + lanes, u);
        // O holds the previous tiles' P V under the old max: rescale it before this tile's P V is issued (S of this
        // tile completing implies the previous P V has completed: one issuing thread, in order)
        if (t > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(tmem + lanes + 192 + 32 * c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= f;
            tmem_st32f(tmem + lanes + 192 + 32 * c, o);
          }
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&bars->o_done, 0, p.err))) {
      tc_fence_after();
      if (!idle) {
        float o[64];
        tmem_ld32p(tmem + lanes + 192, o);
        tmem_ld32p(tmem + lanes + 224, o + 32);
        if (active) {
          const float inv = 1.f / l;
          __nv_bfloat16* dst = p.out + (size_t)(w.q_row + row) * p.ldo + h * kD;
#pragma unroll
          for (int v = 0; v < kD / 8; ++v) {
            uint4 q;
            q.x = pack_bf16x2(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
            q.y = pack_bf16x2(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
            q.z = pack_bf16x2(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
            q.w = pack_bf16x2(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
            reinterpret_cast<uint4*>(dst)[v] = q;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kRTmem);
  }
}

// ---------------------------------------------------------------- relative-position table
// Tiled fp32 product: a block computes 32 table rows x 128 columns; pe rows are made on the fly in shared memory.
__global__ void __launch_bounds__(256) k_pos_table(const float* __restrict__ w, int H, int max_frames, float lw,
                                                   __nv_bfloat16* __restrict__ pos) {
  __shared__ float pe[32][33];
  __shared__ float ws[128][33];
  const int rows = 2 * max_frames - 1;
  const int r0 = blockIdx.x * 32, n0 = blockIdx.y * 128;
  const int tr = threadIdx.x / 32, tc = threadIdx.x % 32;  // 8 x 32 threads: rows tr + 8 i, columns tc + 32 j
  float acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += 32) {
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {
      const int rr = i / 32, kk = i % 32;
      const float r = (float)(r0 + rr - (max_frames - 1));
      const int k = k0 + kk;
      const float wm = expf((float)(k & ~1) * lw);  // w_m = max_period^(-2m / H), k = 2m or 2m + 1
      const float a = r * wm;
      pe[rr][kk] = (k & 1) ? cosf(a) : sinf(a);
    }
    for (int i = threadIdx.x; i < 128 * 32; i += 256) {
      const int nn = i / 32, kk = i % 32;
      ws[nn][kk] = (n0 + nn < H) ? w[(size_t)(n0 + nn) * H + k0 + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < 32; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(pe[tr + 8 * i][kk], ws[tc + 32 * j][kk], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = r0 + tr + 8 * i, n = n0 + tc + 32 * j;
      if (r < rows && n < H) pos[(size_t)r * H + n] = __float2bfloat16(acc[i][j]);
    }
}

// ---------------------------------------------------------------- row kernels
// One warp per row; NV float4 per lane (C = 128 NV).
template <int NV>
__global__ void __launch_bounds__(256) k_enc_ln(const float* x, const float* __restrict__ w, const float* __restrict__ b,
                                                float eps, int rows, float* out_f32, __nv_bfloat16* out_bf16,
                                                const uint8_t* __restrict__ pad) {
  constexpr int C = 128 * NV;
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const bool zero = pad && pad[r];
  float4 v[NV];
  const float4* src = reinterpret_cast<const float4*>(x + (size_t)r * C);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = src[lane + 32 * i];
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(sum) * (1.f / C);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i].x -= mean;
    v[i].y -= mean;
    v[i].z -= mean;
    v[i].w -= mean;
    sq += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
  }
  const float rstd = rsqrtf(warp_sum(sq) * (1.f / C) + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = 4 * (lane + 32 * i);
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + c)), bb = __ldg(reinterpret_cast<const float4*>(b + c));
    float4 y;
    y.x = zero ? 0.f : fmaf(v[i].x * rstd, ww.x, bb.x);
    y.y = zero ? 0.f : fmaf(v[i].y * rstd, ww.y, bb.y);
    y.z = zero ? 0.f : fmaf(v[i].z * rstd, ww.z, bb.z);
    y.w = zero ? 0.f : fmaf(v[i].w * rstd, ww.w, bb.w);
    if (out_f32) reinterpret_cast<float4*>(out_f32 + (size_t)r * C)[lane + 32 * i] = y;
    if (out_bf16) {
      uint2 q;
      q.x = pack_bf16x2(y.x, y.y);
      q.y = pack_bf16x2(y.z, y.w);
      reinterpret_cast<uint2*>(out_bf16 + (size_t)r * C)[lane + 32 * i] = q;
    }
  }
}

__global__ void __launch_bounds__(256) k_embed_rows(const __nv_bfloat16* __restrict__ emb, const int* __restrict__ tok,
                                                    int rows, int C, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int t = tok[r];
  const int n16 = C / 8;  // 16-byte chunks per row
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)r * C);
  const uint4* src = reinterpret_cast<const uint4*>(emb + (size_t)(t < 0 ? 0 : t) * C);
  for (int i = lane; i < n16; i += 32) dst[i] = t < 0 ? make_uint4(0, 0, 0, 0) : __ldg(src + i);
}

// One block per window; 16-byte chunks.
__global__ void __launch_bounds__(256) k_pl_cache(__nv_bfloat16* o, int C, const EncRow* __restrict__ rows,
                                                  __nv_bfloat16* cache, int cache_frames) {
  extern __shared__ uint4 old[];  // the window's 2 cached frames
  pdl_wait();
  pdl_launch();
  const EncRow e = rows[blockIdx.x];
  const int n16 = C / 8;
  uint4* cf = reinterpret_cast<uint4*>(cache + (size_t)e.cache * cache_frames * C);  // frames 0, 1: this cache
  for (int i = threadIdx.x; i < 2 * n16; i += blockDim.x) old[i] = cf[i];
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * n16; i += blockDim.x)
    reinterpret_cast<uint4*>(o + (size_t)(e.seg1 + i / n16) * C)[i % n16] = old[i];
  // new cache: frames T, T + 1 of [cache | o]: the old cache's frames while T + f < 2, else o's rows
  for (int i = threadIdx.x; i < 2 * n16; i += blockDim.x) {
    const int f = i / n16, c = i % n16, x = e.T + f;
    cf[i] = x < 2 ? old[x * n16 + c] : reinterpret_cast<const uint4*>(o + (size_t)(e.seg1 + x) * C)[c];
  }
}

__global__ void __launch_bounds__(256) k_up_pack(const float* __restrict__ h, int C, const EncRow* __restrict__ rows,
                                                 __nv_bfloat16* u, __nv_bfloat16* cache, int cache_frames) {
  extern __shared__ uint4 old[];  // the window's 4 cached upsampled frames
  pdl_wait();
  pdl_launch();
  const EncRow e = rows[blockIdx.x];
  const int n16 = C / 8;
  uint4* cf = reinterpret_cast<uint4*>(cache + ((size_t)e.cache * cache_frames + 2) * C);  // frames 2 .. 5
  for (int i = threadIdx.x; i < 4 * n16; i += blockDim.x) old[i] = cf[i];
  __syncthreads();
  // frame x of [cache | upsampled] as 8 bf16
  auto frame = [&](int x, int c) -> uint4 {
    if (x < 4) return old[x * n16 + c];
    const float4* src = reinterpret_cast<const float4*>(h + (size_t)(e.seg1 + 2 + (x - 4) / 2) * C) + 2 * c;
    const float4 a = src[0], b = src[1];
    return make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  };
  const int nf = 4 + 2 * e.T;
  for (int i = threadIdx.x; i < nf * n16; i += blockDim.x)
    reinterpret_cast<uint4*>(u + (size_t)(e.seg2 + i / n16) * C)[i % n16] = frame(i / n16, i % n16);
  for (int i = threadIdx.x; i < 4 * n16; i += blockDim.x) cf[i] = frame(2 * e.T + i / n16, i % n16);
}

// One warp per new key: 2 H bf16 ([k | v]) = H / 4 16-byte chunks.
__global__ void __launch_bounds__(256) k_enc_kv_scatter(const __nv_bfloat16* __restrict__ qkv4, int H,
                                                        const int* __restrict__ row, const int* __restrict__ slot, int n,
                                                        __nv_bfloat16* __restrict__ pool) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= n) return;
  const uint4* src = reinterpret_cast<const uint4*>(qkv4 + (size_t)row[i] * 4 * H + 2 * H);
  uint4* dst = reinterpret_cast<uint4*>(pool + (size_t)slot[i] * 2 * H);
  for (int c = lane; c < H / 4; c += 32) dst[c] = __ldg(src + c);
}

__global__ void __launch_bounds__(256) k_gather_rows_f32(const float* __restrict__ src, int C, const int* __restrict__ row,
                                                         int n, float* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= n) return;
  const float4* s = reinterpret_cast<const float4*>(src + (size_t)row[i] * C);
  float4* d = reinterpret_cast<float4*>(out + (size_t)i * C);
  for (int c = lane; c < C / 4; c += 32) d[c] = __ldg(s + c);
}

inline int ck(cudaError_t e) {
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace

bool make_relattn_tmaps(CUtensorMap* tm_q, CUtensorMap* tm_pos, const void* qkv4, int rows, int H, const void* pos,
                        int max_frames) {
  return make_tmap_2d(tm_q, qkv4, 2, (uint64_t)rows, (uint64_t)4 * H, (uint64_t)8 * H, kRQ, kD) &&
         make_tmap_2d(tm_pos, pos, 2, (uint64_t)(2 * max_frames - 1), (uint64_t)H, (uint64_t)2 * H, kRBox, kD);
}

int launch_relattn(const RelArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_pos, cudaStream_t st) {
  if (a.n_work <= 0) return T2W_OK;
  if (!a.work || !a.pool || !a.kv_idx || !a.out || a.heads <= 0 || a.pool_ld != 2 * a.heads * kD || a.ldo % 8)
    return T2W_ERR_INVALID;
  static std::atomic<uint64_t> attr_done{0};
  if (const int rc = ck(smem_attr_once(k_relattn, kRSmem, attr_done))) return rc;
  return ck(launch_k(k_relattn, dim3(a.n_work * a.heads), dim3(kRThreads), kRSmem, st, tm_q, tm_pos, a));
}

int launch_pos_table(const float* w, int H, int max_frames, float max_period, __nv_bfloat16* pos, cudaStream_t st) {
  if (!w || !pos || H <= 0 || H % 32 || max_frames <= 0) return T2W_ERR_INVALID;
  const int rows = 2 * max_frames - 1;
  const float lw = -logf(max_period) / (float)H;
  dim3 grid((rows + 31) / 32, (H + 127) / 128);
  k_pos_table<<<grid, 256, 0, st>>>(w, H, max_frames, lw, pos);
  return ck(cudaGetLastError());
}

int launch_enc_ln(const float* x, const float* w, const float* b, float eps, int rows, int C, float* out_f32,
                  __nv_bfloat16* out_bf16, const uint8_t* pad, cudaStream_t st) {
  if (rows <= 0) return T2W_OK;
  if (!x || !w || !b || C % 128 || C > 1024 || (!out_f32 && !out_bf16)) return T2W_ERR_INVALID;
  const dim3 grid((rows + 7) / 8);
  switch (C / 128) {
    case 1: return ck(launch_k(k_enc_ln<1>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 2: return ck(launch_k(k_enc_ln<2>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 3: return ck(launch_k(k_enc_ln<3>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 4: return ck(launch_k(k_enc_ln<4>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 5: return ck(launch_k(k_enc_ln<5>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 6: return ck(launch_k(k_enc_ln<6>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    case 7: return ck(launch_k(k_enc_ln<7>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
    default: return ck(launch_k(k_enc_ln<8>, grid, dim3(256), 0, st, x, w, b, eps, rows, out_f32, out_bf16, pad));
  }
}

int launch_embed_rows(const __nv_bfloat16* emb, const int* tok, int rows, int C, __nv_bfloat16* out, cudaStream_t st) {
  if (rows <= 0) return T2W_OK;
  if (!emb || !tok || !out || C % 8) return T2W_ERR_INVALID;
  return ck(launch_k(k_embed_rows, dim3((rows + 7) / 8), dim3(256), 0, st, emb, tok, rows, C, out));
}

int launch_pl_cache(__nv_bfloat16* o, int C, const EncRow* rows, int n, __nv_bfloat16* cache, int cache_frames,
                    cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  if (!o || !rows || !cache || C % 8) return T2W_ERR_INVALID;
  return ck(launch_k(k_pl_cache, dim3(n), dim3(256), (size_t)2 * C * 2, st, o, C, rows, cache, cache_frames));
}

int launch_up_pack(const float* h, int C, const EncRow* rows, int n, __nv_bfloat16* u, __nv_bfloat16* cache,
                   int cache_frames, cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  if (!h || !rows || !u || !cache || C % 8) return T2W_ERR_INVALID;
  return ck(launch_k(k_up_pack, dim3(n), dim3(256), (size_t)4 * C * 2, st, h, C, rows, u, cache, cache_frames));
}

int launch_enc_kv_scatter(const __nv_bfloat16* qkv4, int H, const int* row, const int* slot, int n, __nv_bfloat16* pool,
                          cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  if (!qkv4 || !row || !slot || !pool || H % 4) return T2W_ERR_INVALID;
  return ck(launch_k(k_enc_kv_scatter, dim3((n + 7) / 8), dim3(256), 0, st, qkv4, H, row, slot, n, pool));
}

int launch_gather_rows_f32(const float* src, int C, const int* row, int n, float* out, cudaStream_t st) {
  if (n <= 0) return T2W_OK;
  if (!src || !row || !out || C % 4) return T2W_ERR_INVALID;
  return ck(launch_k(k_gather_rows_f32, dim3((n + 7) / 8), dim3(256), 0, st, src, C, row, n, out));
}

}  // namespace t2w
