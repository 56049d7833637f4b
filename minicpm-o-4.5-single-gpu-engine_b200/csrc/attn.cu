// Varlen attention over packed [prompt | chunk] sequences, head_dim 64, on tcgen05 tensor cores.
//
// One CTA per (128-query tile, head).  Mask (the reference's streaming form, packed): a query at position i of its
// sequence attends keys j < lim(i), lim = P for prompt queries (i < P), L for chunk queries.  The reference solves the
// prompt alone and then the chunk against the prompt's cached keys (engine/runtime/token2wav_batch.py:632-702,
// FlashInfer non-causal prefill over [new, cache] slots: engine/runtime/dit_fast.py:347-367); attention depends only on
// the key set, so both give the same rows.
//
// Warps: 0 = TMA (Q once, K/V tiles of 128 keys, 2 stages), 1 = MMA issuer, 2-5 = softmax / output, one query row per
// thread (TMEM lane).  Per key tile j: S = Q K^T (M 128, N 128, K 64) into TMEM; the row's thread reads S, updates its
// running max / sum, writes P = exp(S - m) as bf16 into shared memory (K-major, 128B swizzle), then O_j = P V (M 128,
// N 64, K 128, V read MN-major straight from its TMA tile) into TMEM; the thread folds O_j into its fp32 register
// accumulator with the running rescale.  No TMA multicast.
#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kTile = 128;
constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int kSCol = 0, kOCol = 128, kTmemCols = 256;
constexpr int kSmem = kTileBytes * (1 + 2 + 2 + 2) + 1024 + 256;  // Q, K x2, V x2, P (2 swizzle atoms)

struct DevArgs {
  const AttnWork* work;
  int heads;
  __nv_bfloat16* out;
  int ldo;
  float scale_log2;
  int* err;
};

__global__ void __launch_bounds__(192, 1) k_attn(const __grid_constant__ CUtensorMap tm, const DevArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;      // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;  // 2 stages
  uint8_t* sP = sV + 2 * kTileBytes;  // keys 0..63 | keys 64..127
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_full = bars + 8;
  uint64_t* o_free = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const AttnWork w = p.work[blockIdx.x];
  const int h = blockIdx.y;
  const int H = p.heads * kD;
  const int kmax = (w.q_pos + kTile > w.P) ? w.L : w.P;  // any chunk query in the tile sees every key
  const int n_kt = (kmax + kTile - 1) / kTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(o_free, 4);
    fence_mbar_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tm, h * kD, w.q_row, q_full);
      for (int j = 0; j < n_kt; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1u, p.err)) break;
        mbar_expect_tx(&kv_full[s], 2 * kTileBytes);
        tma_load_2d(sK + s * kTileBytes, &tm, H + h * kD, w.k_row + j * kTile, &kv_full[s]);
        tma_load_2d(sV + s * kTileBytes, &tm, 2 * H + h * kD, w.k_row + j * kTile, &kv_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(kTile, kTile);
      constexpr uint32_t idesc_pv = idesc_bf16(kTile, kD, /*b_mn_major=*/true);
      bool ok = mbar_wait(q_full, 0, p.err);
      const uint32_t q0 = smem_u32(sQ), p0 = smem_u32(sP);
      for (int j = 0; j < n_kt && ok; ++j) {
        const int s = j & 1;
        if (!(ok = mbar_wait(&kv_full[s], (j >> 1) & 1, p.err))) break;
        if (j > 0 && !(ok = mbar_wait(s_free, (j - 1) & 1, p.err))) break;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sK + s * kTileBytes), v0 = smem_u32(sV + s * kTileBytes);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_f16(tmem + kSCol, sdesc_sw128(q0 + 32 * k, 1024, 16), sdesc_sw128(k0 + 32 * k, 1024, 16), idesc_qk,
                   k ? 1u : 0u);
        umma_commit(s_full);
        if (!(ok = mbar_wait(p_full, j & 1, p.err))) break;
        if (j > 0 && !(ok = mbar_wait(o_free, (j - 1) & 1, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          // A = P (K-major): 16 keys at byte 32 (k % 4) of swizzle atom k / 4.  B = V (MN-major): 16 key rows.
          umma_f16(tmem + kOCol, sdesc_sw128(p0 + (k >> 2) * kTileBytes + 32 * (k & 3), 1024, 16),
                   sdesc_sw128(v0 + k * 16 * 128, 1024, 8192), idesc_pv, k ? 1u : 0u);
        }
        umma_commit(o_full);
        umma_commit(&kv_empty[s]);
      }
    }
  } else {
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // query row of the tile == TMEM lane
    const int pos = w.q_pos + r;
    const int lim = pos < w.P ? w.P : (pos < w.L ? w.L : 0);
    const uint32_t trow = tmem + ((uint32_t)(qw * 32) << 16);
    float m = -INFINITY, l = 0.f;
    float o[kD];
#pragma unroll
    for (int i = 0; i < kD; ++i) o[i] = 0.f;
    uint8_t* prow = sP + r * 128;
    for (int j = 0; j < n_kt; ++j) {
      // warp-uniform: tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, j & 1, p.err))) break;
      tc_fence_after();
      const int kb = j * kTile;
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(trow + kSCol + 32 * c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (kb + 32 * c + i < lim) mx = fmaxf(mx, v[i]);
      }
      const float m_new = fmaxf(m, mx * p.scale_log2);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(trow + kSCol + 32 * c, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k0 = kb + 32 * c + 2 * i;
          const float e0 = (k0 < lim) ? exp2f(v[2 * i] * p.scale_log2 - m_use) : 0.f;
          const float e1 = (k0 + 1 < lim) ? exp2f(v[2 * i + 1] * p.scale_log2 - m_use) : 0.f;
          rs += e0 + e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        // keys 32c .. 32c + 31 = four 16-byte chunks of the row, in atom (32c / 64), swizzled by row % 8
        uint8_t* atom = prow + (c >> 1) * kTileBytes;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = ((c & 1) * 4 + u) ^ (r & 7);
          *reinterpret_cast<uint4*>(atom + chunk * 16) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(s_free);
        mbar_arrive(p_full);
      }
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_use);
      l = l * alpha + rs;
      m = m_new;
      if (!__all_sync(0xffffffffu, mbar_wait(o_full, j & 1, p.err))) break;
      tc_fence_after();
      float oj[32];
      tmem_ld32(trow + kOCol, oj);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], alpha, oj[i]);
      tmem_ld32(trow + kOCol + 32, oj);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[32 + i] = fmaf(o[32 + i], alpha, oj[i]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
    }
    if (lim > 0) {
      const float inv = 1.f / l;
      __nv_bfloat16* dst = p.out + (size_t)(w.q_row + r) * p.ldo + h * kD;
#pragma unroll
      for (int u = 0; u < kD / 8; ++u) {
        uint4 q;
        q.x = pack_bf16x2(o[8 * u + 0] * inv, o[8 * u + 1] * inv);
        q.y = pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv);
        q.z = pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv);
        q.w = pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv);
        reinterpret_cast<uint4*>(dst)[u] = q;
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
  DevArgs p{a.work, a.heads, reinterpret_cast<__nv_bfloat16*>(a.out), a.heads * kD, a.scale_log2, a.err};
  dim3 grid(a.n_work, a.heads);
  k_attn<<<grid, 192, kSmem, st>>>(*tm, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace t2w
