// Varlen attention over packed [prompt | chunk] sequences, head_dim 64, on tcgen05 tensor cores.
//
// Mask (the reference's streaming form, packed): a query at position i of its sequence attends keys j < lim(i),
// lim = P for prompt queries (i < P), L for chunk queries.  The reference solves the prompt alone and then the chunk
// against the prompt's cached keys (engine/runtime/token2wav_batch.py:632-702, FlashInfer non-causal prefill over
// [new, cache] slots: engine/runtime/dit_fast.py:347-367); attention depends only on the key set, so both give the
// same rows.
//
// Persistent CTAs (one per SM), two independent pipelines per CTA.  A work item is (128-query tile, head); pipeline p
// of CTA c takes items p + 2 (c + k * grid).  Warps: 0 = TMA producer for both pipelines, 1 = TMEM allocator and MMA
// issuer for both (each a polling loop over the two pipelines' barriers), 2-5 = softmax of pipeline 0, 6-9 = softmax of
// pipeline 1 (one query row per thread = TMEM lane).  Per key tile j of 128 keys:
//   S = Q K^T (M 128, N 128, K 64) into the pipeline's TMEM S region;
//   the row's thread loads its 128 scores, updates the running max (log2 domain) and, when that max rises by more than
//   8 (or on the first tile), rescales its O row in TMEM; it writes P = 2^(S c - m) as bf16 pairs back into the S
//   columns (tcgen05.st), so the P V product reads A straight from TMEM;
//   O += P V (M 128, N 64, K 128, V MN-major from its TMA tile) accumulates in the pipeline's TMEM O region.
// Tensor-core ops of one issuing thread run in issue order, so S_{j+1} never overwrites P_j before P_j V_j has read it.
// No TMA multicast.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kTile = 128;
constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int kStages = 2;
constexpr int kPipeBytes = kTileBytes * (1 + 2 * kStages);  // Q + K/V ring
constexpr int kSmem = 2 * kPipeBytes + 1024 + 512;
constexpr int kTmemCols = 512;  // per pipeline: S/P 128 columns at 256 p, O 64 columns at 256 p + 128
constexpr float kRescaleThreshold = 8.f;

struct DevArgs {
  const AttnWork* work;
  int n_items, heads;
  __nv_bfloat16* out;
  int ldo;
  float scale_log2;
  int* err;
};

struct PipeBars {
  uint64_t q_full, q_free, kv_full[kStages], kv_empty[kStages], s_full, p_full, o_done, o_free;
};

T2W_DEV void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
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

// 32 lanes x 64 columns, no wait (the caller waits once for several loads).
T2W_DEV void tmem_ld64_nowait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
T2W_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// O (+)= P V with P from TMEM (A operand, K-major: 2 bf16 keys per 32-bit column) and V from shared memory.
T2W_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

T2W_DEV int item_tiles(const AttnWork& w) {
  const int kmax = (w.q_pos + kTile > w.P) ? w.L : w.P;  // any chunk query in the tile sees every key
  return (kmax + kTile - 1) / kTile;
}

// Per-pipeline progress of the producer and of the MMA issuer (each a polling state machine).
struct ProdState {
  int k = 0, item = -1, j = 0, n_kt = 0, stage = 0;
  uint32_t phase = 0;
  bool need_q = true, done = false;
  AttnWork w{};
  int h = 0;
};
struct MmaState {
  int k = 0, item = -1, j = 0, n_kt = 0, stage = 0, tiles = 0;
  uint32_t phase = 0;
  int st = 0;  // 0 wait Q, 1 wait K/V, 2 wait P, 3 done
  bool done = false;
};

__global__ void __launch_bounds__(320, 1) k_attn(const __grid_constant__ CUtensorMap tm, const DevArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PipeBars* bars = reinterpret_cast<PipeBars*>(smem + 2 * kPipeBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.heads * kD;

  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q) {
      PipeBars& b = bars[q];
      mbar_init(&b.q_full, 1);
      mbar_init(&b.q_free, 1);
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&b.kv_full[s], 1);
        mbar_init(&b.kv_empty[s], 1);
      }
      mbar_init(&b.s_full, 1);
      mbar_init(&b.p_full, 4);
      mbar_init(&b.o_done, 1);
      mbar_init(&b.o_free, 4);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm);
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
  const int stride = 2 * gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      ProdState ps[2];
      long long idle_since = clock64();
      uint32_t polls = 0;
      bool abort = false;
      while (!(ps[0].done && ps[1].done) && !abort) {
        bool progressed = false;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          ProdState& s = ps[q];
          if (s.done) continue;
          PipeBars& b = bars[q];
          uint8_t* base = smem + q * kPipeBytes;
          if (s.need_q) {
            const int item = q + 2 * blockIdx.x + s.k * stride;
            if (item >= p.n_items) {
              s.done = true;
              progressed = true;
              continue;
            }
            // the previous item's last S MMA has read the Q buffer
            if (!mbar_test(smem_u32(&b.q_free), ((s.k & 1) ^ 1u))) continue;
            s.item = item;
            s.w = p.work[item / p.heads];
            s.h = item % p.heads;
            s.n_kt = item_tiles(s.w);
            s.j = 0;
            mbar_expect_tx(&b.q_full, kTileBytes);
            tma_load_2d(base, &tm, s.h * kD, s.w.q_row, &b.q_full);
            s.need_q = false;
            progressed = true;
          } else {
            if (!mbar_test(smem_u32(&b.kv_empty[s.stage]), s.phase ^ 1u)) continue;
            uint8_t* kv = base + kTileBytes + s.stage * 2 * kTileBytes;
            mbar_expect_tx(&b.kv_full[s.stage], 2 * kTileBytes);
            tma_load_2d(kv, &tm, H + s.h * kD, s.w.k_row + s.j * kTile, &b.kv_full[s.stage]);
            tma_load_2d(kv + kTileBytes, &tm, 2 * H + s.h * kD, s.w.k_row + s.j * kTile, &b.kv_full[s.stage]);
            if (++s.stage == kStages) {
              s.stage = 0;
              s.phase ^= 1u;
            }
            if (++s.j == s.n_kt) {
              s.need_q = true;
              ++s.k;
            }
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = clock64();
        } else if ((++polls & 255u) == 0 && clock64() - idle_since > kWaitLimitCycles) {
          atomicExch(p.err, T2W_ERR_TIMEOUT);
          abort = true;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(kTile, kTile);
      constexpr uint32_t idesc_pv = idesc_bf16(kTile, kD, /*b_mn_major=*/true);
      MmaState ms[2];
      long long idle_since = clock64();
      uint32_t polls = 0;
      bool abort = false;
      while (!(ms[0].done && ms[1].done) && !abort) {
        bool progressed = false;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          MmaState& s = ms[q];
          if (s.done) continue;
          PipeBars& b = bars[q];
          uint8_t* base = smem + q * kPipeBytes;
          const uint32_t sreg = tmem + 256 * q, oreg = sreg + 128;
          if (s.st == 0) {  // wait for this item's Q
            const int item = q + 2 * blockIdx.x + s.k * stride;
            if (item >= p.n_items) {
              s.done = true;
              progressed = true;
              continue;
            }
            if (!mbar_test(smem_u32(&b.q_full), s.k & 1)) continue;
            s.item = item;
            s.n_kt = item_tiles(p.work[item / p.heads]);
            s.j = 0;
            s.st = 1;
            progressed = true;
          } else if (s.st == 1) {  // S_j = Q K_j^T
            if (!mbar_test(smem_u32(&b.kv_full[s.stage]), s.phase)) continue;
            tc_fence_after();
            const uint32_t q0 = smem_u32(base), k0 = smem_u32(base + kTileBytes + s.stage * 2 * kTileBytes);
#pragma unroll
            for (int k = 0; k < kD / 16; ++k)
              umma_f16(sreg, sdesc_sw128(q0 + 32 * k, 1024, 16), sdesc_sw128(k0 + 32 * k, 1024, 16), idesc_qk, k ? 1u : 0u);
            umma_commit(&b.s_full);
            if (s.j == s.n_kt - 1) umma_commit(&b.q_free);
            s.st = 2;
            progressed = true;
          } else {  // O += P_j V_j once the softmax has written P_j (and, for j = 0, read the previous item's O)
            if (!mbar_test(smem_u32(&b.p_full), s.tiles & 1)) continue;
            if (s.j == 0 && s.k > 0 && !mbar_test(smem_u32(&b.o_free), (s.k - 1) & 1)) continue;
            tc_fence_after();
            const uint32_t v0 = smem_u32(base + kTileBytes + s.stage * 2 * kTileBytes + kTileBytes);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k)
              umma_f16_ts(oreg, sreg + 8 * k, sdesc_sw128(v0 + k * 16 * 128, 1024, 8192), idesc_pv,
                          (s.j > 0 || k > 0) ? 1u : 0u);
            umma_commit(&b.o_done);
            umma_commit(&b.kv_empty[s.stage]);
            ++s.tiles;
            if (++s.stage == kStages) {
              s.stage = 0;
              s.phase ^= 1u;
            }
            if (++s.j == s.n_kt) {
              ++s.k;
              s.st = 0;
            } else {
              s.st = 1;
            }
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = clock64();
        } else if ((++polls & 255u) == 0 && clock64() - idle_since > kWaitLimitCycles) {
          atomicExch(p.err, T2W_ERR_TIMEOUT);
          abort = true;
        }
      }
    }
  } else {
    const int q = (warp - 2) >> 2;  // pipeline
    const int qw = warp & 3;        // TMEM lane quarter
    const int r = qw * 32 + lane;   // query row of the tile
    PipeBars& b = bars[q];
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    const uint32_t sreg = tmem + 256 * q + lanes, oreg = tmem + 256 * q + 128 + lanes;
    int tiles = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int item = q + 2 * blockIdx.x + k * stride;
      if (item >= p.n_items) break;
      const AttnWork w = p.work[item / p.heads];
      const int h = item % p.heads;
      const int n_kt = item_tiles(w);
      const int pos = w.q_pos + r;
      const int lim = pos < w.P ? w.P : (pos < w.L ? w.L : 0);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kt; ++j, ++tiles) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b.s_full, tiles & 1, p.err)))) break;
        // P_{j-1} V_{j-1} was issued before S_j, so it is complete too; waiting keeps o_done's phases in step
        if (j > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(&b.o_done, (tiles - 1) & 1, p.err)))) break;
        tc_fence_after();
        // all 128 scores of the row in one TMEM round trip
        uint32_t sr[128];
        tmem_ld64_nowait(sreg, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
        tmem_ld64_nowait(sreg + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
        tmem_ld_wait();
        const int kb = j * kTile;
        // rows whose 128 keys of this tile are all valid skip the mask (every prompt row before the prompt's last
        // tile, every chunk row before the sequence's last tile)
        const bool full = __all_sync(0xffffffffu, kb + kTile <= lim);
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int i = 0; i < kTile; i += 2) mx = fmaxf(mx, fmaxf(__uint_as_float(sr[i]), __uint_as_float(sr[i + 1])));
        } else {
#pragma unroll
          for (int i = 0; i < kTile; ++i)
            if (kb + i < lim) mx = fmaxf(mx, __uint_as_float(sr[i]));
        }
        mx *= p.scale_log2;
        // raise the reference max only when it grows by more than the threshold (p <= 2^8 fits bf16 comfortably)
        const bool raise = mx > m + kRescaleThreshold;
        const float m_old = m;
        m = raise ? mx : m;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        // P = 2^(S c - m) as bf16 pairs, written back over the S columns (each pair replaces two consumed scores)
        const float2 c2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_use, -m_use);
        float2 rs2 = make_float2(0.f, 0.f);
        uint32_t u[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 a = fma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), c2, nm2);
          float2 e = make_float2(exp2_approx(a.x), exp2_approx(a.y));
          if (!full) {
            const int kk = kb + 2 * i;
            e.x = (kk < lim) ? e.x : 0.f;
            e.y = (kk + 1 < lim) ? e.y : 0.f;
          }
          rs2 = add2(rs2, e);
          u[i] = pack_bf16x2(e.x, e.y);
        }
        const float rs = rs2.x + rs2.y;
        tmem_st32(sreg, *reinterpret_cast<const uint32_t(*)[32]>(&u[0]));
        tmem_st32(sreg + 32, *reinterpret_cast<const uint32_t(*)[32]>(&u[32]));
        // O holds P_{<j} V_{<j} relative to the old reference max: rescale it (rare) before P_j V_j is issued
        if (j > 0 && __any_sync(0xffffffffu, raise)) {
          const float f = raise ? exp2_approx(m_old - m) : 1.f;
          l *= f;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(oreg + 32 * c, o);
            uint32_t ou[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) ou[i] = __float_as_uint(o[i] * f);
            tmem_st32(oreg + 32 * c, ou);
          }
        }
        l += rs;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b.p_full);
      }
      if (!ok) break;
      // the item's last P V
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b.o_done, (tiles - 1) & 1, p.err)))) break;
      tc_fence_after();
      float o[kD];
      tmem_ld32p(oreg, o);
      tmem_ld32p(oreg + 32, o + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b.o_free);
      if (lim > 0) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = p.out + (size_t)(w.q_row + r) * p.ldo + h * kD;
#pragma unroll
        for (int u = 0; u < kD / 8; ++u) {
          uint4 v;
          v.x = pack_bf16x2(o[8 * u + 0] * inv, o[8 * u + 1] * inv);
          v.y = pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv);
          v.z = pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv);
          v.w = pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv);
          reinterpret_cast<uint4*>(dst)[u] = v;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int launch_attn(const AttnArgs& a, cudaStream_t st, const CUtensorMap* tm) {
  if (!a.qkv || !a.work || !a.out || a.rows <= 0 || a.heads <= 0 || a.n_work < 0) return T2W_ERR_INVALID;
  if (a.n_work == 0) return T2W_OK;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
    attr_done = true;
  }
  CUtensorMap m;
  if (!tm) {
    const uint64_t cols = 3ull * a.heads * kD;
    if (!make_tmap_2d(&m, a.qkv, 2, (uint64_t)a.rows, cols, cols * 2, kTile, kD)) return T2W_ERR_INVALID;
    tm = &m;
  }
  const int n_items = a.n_work * a.heads;
  DevArgs p{a.work, n_items, a.heads, reinterpret_cast<__nv_bfloat16*>(a.out), a.heads * kD, a.scale_log2, a.err};
  int grid = (n_items + 1) / 2;
  if (grid > num_sms()) grid = num_sms();
  cudaError_t e = launch_k(k_attn, dim3(grid), dim3(320), kSmem, st, *tm, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace t2w

// ---------------------------------------------------------------------------------------------------------------------
// Allocation-free attention entry point.
//
// Some callers cannot allocate device memory at the moment they call in: a serving runtime that reserves every byte
// of the GPU up front for its own pool (a cudaMalloc there fails or breaks its memory accounting), or a plugin that is
// invoked inside a host framework's region where calling the CUDA allocator is not permitted.  t2w_attn_varlen needs a
// small device-side work list (one entry per 128-query tile), which it allocates per call; this variant keeps that
// list in a fixed file-scope device array instead.  The array is reserved in every GPU that loads this library and is
// held until the process exits.
namespace {

constexpr int kNoAllocMaxWork = 8192;  // query tiles (of 128 rows) per call: 8192 x 20 B = 160 KB per GPU
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) t2w::AttnWork g_noalloc_work[kNoAllocMaxWork];

std::mutex g_noalloc_mu;
t2w::AttnWork* g_noalloc_ptr[kNoAllocMaxDevices] = {};

}  // namespace

extern "C" int t2w_attn_varlen_noalloc(const void* qkv, int32_t rows, int32_t heads, int32_t n_seq, const int32_t* seq_row,
                                       const int32_t* seq_len, const int32_t* prompt_len, void* out, void* stream) {
  using namespace t2w;
  if (!qkv || !out || !seq_row || !seq_len || !prompt_len || n_seq < 0 || heads <= 0) return T2W_ERR_INVALID;
  std::vector<AttnWork> work;
  for (int s = 0; s < n_seq; ++s) {
    if (seq_len[s] <= 0 || prompt_len[s] < 0 || prompt_len[s] > seq_len[s] || seq_row[s] < 0 ||
        seq_row[s] + seq_len[s] > rows)
      return T2W_ERR_INVALID;
    for (int q = 0; q < seq_len[s]; q += 128) work.push_back(AttnWork{seq_row[s] + q, seq_row[s], q, prompt_len[s], seq_len[s]});
  }
  if (work.size() > (size_t)kNoAllocMaxWork) return T2W_ERR_INVALID;  // beyond the fixed scratch array
  if (work.empty()) return T2W_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    if (e != cudaSuccess) set_cuda_error(e);
    return e != cudaSuccess ? T2W_ERR_CUDA : T2W_ERR_UNSUPPORTED;
  }
  AttnWork* scratch = nullptr;
  {
    // once per device, with that device current: the array's device address (its host-side name is only a stand-in)
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_noalloc_work);
      if (e != cudaSuccess) {
        set_cuda_error(e);
        return T2W_ERR_CUDA;
      }
      g_noalloc_ptr[dev] = static_cast<AttnWork*>(ptr);
    }
    scratch = g_noalloc_ptr[dev];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = cudaMemcpyAsync(scratch, work.data(), work.size() * sizeof(AttnWork), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  AttnArgs a;
  a.qkv = qkv;
  a.rows = rows;
  a.heads = heads;
  a.work = scratch;
  a.n_work = (int)work.size();
  a.out = out;
  a.scale_log2 = (float)(1.4426950408889634 / 8.0);
  return launch_attn(a, st);
}
