// Varlen attention over packed [prompt | chunk] sequences, head_dim 64, on tcgen05 tensor cores.
//
// Mask (the reference's streaming form, packed): a query at position i of its sequence attends keys j < lim(i),
// lim = P for prompt queries (i < P), L for chunk queries.  The reference solves the prompt alone and then the chunk
// against the prompt's cached keys (engine/runtime/token2wav_batch.py:632-702, FlashInfer non-causal prefill over
// [new, cache] slots: engine/runtime/dit_fast.py:347-367); attention depends only on the key set, so both give the
// same rows.
//
// Persistent CTAs (one per SM), two independent pipelines per CTA.  A work item is (128-query tile, head); pipeline p
// of CTA c takes items p + 2 (c + k * grid).  Warps: 0 / 1 = TMA producers of pipelines 0 / 1, 2 / 3 = MMA issuers of
// pipelines 0 / 1 (warp 2 also allocates TMEM), 4-7 = softmax of pipeline 0, 8-11 = softmax of pipeline 1 (one query
// row per thread = TMEM lane).  Each control thread serves one pipeline with blocking waits in a fixed order.  Keys go
// in tiles of 64; per tile t of a pipeline:
//   S_t = Q K_t^T (M 128, N 64, K 64) into S buffer t % 2 of the pipeline's TMEM;
//   the row's thread loads its 64 scores, keeps a running max (log2 domain) that it raises only when the tile's max
//   exceeds it by more than 8 (then it rescales its O row in TMEM), and writes P = 2^(S c - m) as bf16 pairs back over
//   the scores (tcgen05.st), so the P V product reads its A operand straight from TMEM;
//   O += P_t V_t (M 128, N 64, K 64, V MN-major from its TMA tile) accumulates in the pipeline's TMEM O region.
// With two S buffers the issuer computes S_{t+1} (and S_{t+2} once P_t V_t is issued) while the softmax works on tile
// t, so the softmax warps run from tile to tile without waiting on the tensor core.  Tensor-core ops of one issuing
// thread run in issue order, so S_{t+2} never overwrites P_t before P_t V_t has read it.  No TMA multicast.
//
// Paired form (gathered keys, every item's queries within 64 rows: the steady-state windows): a pipeline's work item
// is two (query tile, head) items A and B laid out block-diagonally in the same 128-row MMA tiles.  Query rows 0-63
// are A's queries, 64-127 B's (two 64-row TMA boxes); each 64-key tile holds 32 keys of A (smem rows 0-31) and the
// same-numbered 32 keys of B (rows 32-63).  S = Q K^T then holds A x A's keys in rows 0-63 / columns 0-31 and B x B's
// keys in rows 64-127 / columns 32-63; each softmax thread reads its item's 32 columns and writes P for them with
// zeros over the other item's 32, so O = P V takes rows 0-63 from A's values alone and rows 64-127 from B's.  The
// MMA shapes, TMEM regions and barriers are those of the single form; a 50-frame window then keeps all four softmax
// warps busy and a CTA runs four windows' heads at once instead of two.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace t2w {

namespace {

constexpr int kQTile = 128;                    // queries per item
constexpr int kKTile = 64;                     // keys per S tile
constexpr int kD = 64;
constexpr int kQBytes = kQTile * kD * 2;       // 16 KB
constexpr int kKVBytes = kKTile * kD * 2;      // 8 KB each for K and V
// K/V ring per pipeline.  Five stages (two pipelines then take 220 of the 227 KB with the item table) against four:
// target shape 105.6 -> 102.9 ms, steady call of 32 windows 22.8 -> 22.5 ms (the slot pool's gathered keys arrive
// further ahead of their S tiles); config 2 and 64 steady windows unchanged within run-to-run noise.
constexpr int kStages = 5;
constexpr int kPipeBytes = kQBytes + kStages * 2 * kKVBytes;  // 96 KB
constexpr int kMaxCtaItems = 512;  // items per CTA staged in shared memory (the grid grows to keep within it)
constexpr int kPairRows = 64;      // paired form: query rows of each of the two items
constexpr int kPairKeys = 32;      // paired form: keys of each item per 64-key tile
struct ItemEntry {
  AttnWork w;
  int h, n_kt;
  AttnWork w2;  // paired form: item B (h2 = -1 when the pair's second item does not exist)
  int h2;
};
constexpr int kSmem = 2 * kPipeBytes + 1024 + 512 + kMaxCtaItems * (int)sizeof(ItemEntry);
constexpr int kTmemCols = 512;  // pipeline p: S/P buffers at 192 p + {0, 64}, O at 192 p + 128
constexpr float kRescaleThreshold = 8.f;
// The two pipelines of a CTA take consecutive heads of the same query tiles, so left alone they run the same phases at
// the same moments and contend for the same issue slots and special-function units.  Pipeline 1's softmax starts this
// many cycles after its first S tile is ready (about one tile's softmax), and the offset persists because the
// pipelines' items have equal lengths.  Measured on the config-2 solve (16 x 350 frames, 160 launches): attention
// 4.19 -> 3.78 ms per solve; 0.7K / 1.4K / 2.1K / 2.8K / 3.5K / 5.6K cycles gave 4.10 / 4.04 / 3.78 / 3.81 / 3.91 /
// 4.03 ms.
constexpr long long kPipeStagger = 2400;

struct DevArgs {
  const AttnWork* work;
  int n_items, heads;
  int n_flat;       // paired form: (work, head) items; n_items = the pairs
  void* out;        // bf16, or e4m3 with out_sf (the FP8 path's proj input)
  uint8_t* out_sf;  // e4m3 output: UE8M0 scale atoms (one byte per row and 32-column block, sf_offset layout)
  int ldo;
  float scale_log2;
  int* err;
  // gathered keys (slot-pool form): key j of an item is row kv_idx[w.k_row + j] of the pool, K at column h * 64 and V
  // at column heads * 64 + h * 64 of a row of pool_ld bf16
  const __nv_bfloat16* pool;
  const int* kv_idx;
  int pool_ld;
  const void* pf;  // L2 prefetch of the next GEMM's weights, 64 KB per CTA
  unsigned pf_bytes;
};

// 16-byte global -> shared copy (zero-filled when src_bytes == 0) and the arrival of this thread's outstanding copies
// on an mbarrier (counted against the barrier's expected arrivals).
T2W_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
T2W_DEV void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

struct PipeBars {
  uint64_t q_full, q_free, kv_full[kStages], kv_empty[kStages], s_full[2], p_full[2], o_done[2], o_free;
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

// O (+)= P V with P from TMEM (A operand, K-major: 2 bf16 keys per 32-bit column) and V from shared memory.
T2W_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Key tiles of an item.  Packed form: prompt queries see P keys, chunk queries L.  Gathered form (GATHER): the
// window's P queries each see all L keys of the row's list.
template <bool GATHER>
T2W_DEV int item_tiles(const AttnWork& w) {
  const int kmax = GATHER ? w.L : ((w.q_pos + kQTile > w.P) ? w.L : w.P);  // any chunk query in the tile sees every key
  return (kmax + kKTile - 1) / kKTile;
}

template <bool E4M3, bool GATHER, bool PAIR>
__global__ void __launch_bounds__(384, 1) k_attn(const __grid_constant__ CUtensorMap tm_q,
                                                 const __grid_constant__ CUtensorMap tm_kv, const DevArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PipeBars* bars = reinterpret_cast<PipeBars*>(smem + 2 * kPipeBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  ItemEntry* items = reinterpret_cast<ItemEntry*>(smem + 2 * kPipeBytes + 512);  // local item 2 k + q of pipeline q
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.heads * kD;
  const int stride = 2 * gridDim.x;
  // this CTA's items: global item q + 2 (blockIdx.x + k grid) is local item 2 k + q
  const int n_local = (p.n_items > 2 * (int)blockIdx.x) ? ((p.n_items - 2 * (int)blockIdx.x + stride - 1) / stride) * 2 : 0;

  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q) {
      PipeBars& b = bars[q];
      mbar_init(&b.q_full, 1);
      mbar_init(&b.q_free, 1);
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&b.kv_full[s], GATHER ? 32 : 1);  // gathered: one cp.async arrival per producer lane
        mbar_init(&b.kv_empty[s], 1);
      }
      for (int s = 0; s < 2; ++s) {
        mbar_init(&b.s_full[s], 1);
        mbar_init(&b.p_full[s], 4);
        mbar_init(&b.o_done[s], 1);
      }
      mbar_init(&b.o_free, 4);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_kv);
  }
  if (threadIdx.x == 0) prefetch_l2_piece(p.pf, p.pf_bytes, blockIdx.x);
  pdl_wait();
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  for (int i = threadIdx.x; i < n_local && i < kMaxCtaItems; i += blockDim.x) {
    const int item = (i & 1) + 2 * blockIdx.x + (i >> 1) * stride;
    if (item < p.n_items) {
      ItemEntry e;
      if constexpr (PAIR) {
        const int f = 2 * item;
        e.w = p.work[f / p.heads];
        e.h = f % p.heads;
        if (f + 1 < p.n_flat) {
          e.w2 = p.work[(f + 1) / p.heads];
          e.h2 = (f + 1) % p.heads;
        } else {
          e.w2 = e.w;
          e.h2 = -1;
        }
        const int kmax = max(e.w.L, e.h2 >= 0 ? e.w2.L : 0);
        e.n_kt = (kmax + kPairKeys - 1) / kPairKeys;
      } else {
        e.w = p.work[item / p.heads];
        e.h = item % p.heads;
        e.n_kt = item_tiles<GATHER>(e.w);
        e.w2 = e.w;
        e.h2 = -1;
      }
      items[i] = e;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch();
  const uint32_t tmem = *tmem_slot;

  if (warp < 2) {
    const int q = warp;
    PipeBars& b = bars[q];
    uint8_t* base = smem + q * kPipeBytes;
    if constexpr (!GATHER) {
      if (lane == 0) {  // TMA producer of pipeline q
        int t = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
          if (q + 2 * (int)blockIdx.x + k * stride >= p.n_items) break;
          const ItemEntry e = items[2 * k + q];
          // the previous item's last S MMA has read the Q buffer
          if (!(ok = mbar_wait(&b.q_free, (k & 1) ^ 1u, p.err))) break;
          mbar_expect_tx(&b.q_full, kQBytes);
          tma_load_2d(base, &tm_q, e.h * kD, e.w.q_row, &b.q_full);
          for (int j = 0; j < e.n_kt; ++j, ++t) {
            const int st = t % kStages;
            if (!(ok = mbar_wait(&b.kv_empty[st], ((t / kStages) & 1) ^ 1u, p.err))) break;
            uint8_t* kv = base + kQBytes + st * 2 * kKVBytes;
            mbar_expect_tx(&b.kv_full[st], 2 * kKVBytes);
            tma_load_2d(kv, &tm_kv, H + e.h * kD, e.w.k_row + j * kKTile, &b.kv_full[st]);
            tma_load_2d(kv + kKVBytes, &tm_kv, 2 * H + e.h * kD, e.w.k_row + j * kKTile, &b.kv_full[st]);
          }
        }
      }
    } else {
      // gathered K / V: the whole warp copies each 64-key tile from the slot pool with 16-byte cp.async, placing rows
      // in the 128-byte-swizzled layout the TMA tiles have (chunk c of row r at chunk c ^ (r % 8)); keys past the
      // row's list are zero-filled
      int t = 0;
      bool ok = true;
      // The slot indices of the next tile's keys (the next item's first tile after an item's last) are loaded while
      // this tile's copies are issued, so the index load's latency is off the producer's path.
      auto slot_of = [&](const AttnWork& w, int key) { return key < w.L ? __ldg(p.kv_idx + w.k_row + key) : 0; };
      // the key this lane copies into smem row lane + 32 half of tile j, and the item it belongs to (paired form:
      // half 0 = item A's key 32 j + lane, half 1 = item B's key of the same number)
      auto key_of = [&](int j, int half) { return PAIR ? j * kPairKeys + lane : j * kKTile + lane + 32 * half; };
      auto work_of = [&](const ItemEntry& e, int half) -> const AttnWork& { return (PAIR && half) ? e.w2 : e.w; };
      int nxt[2] = {0, 0};
      if (q + 2 * (int)blockIdx.x < p.n_items) {
        nxt[0] = slot_of(work_of(items[q], 0), key_of(0, 0));
        nxt[1] = slot_of(work_of(items[q], 1), key_of(0, 1));
      }
      for (int k = 0; ok; ++k) {
        if (q + 2 * (int)blockIdx.x + k * stride >= p.n_items) break;
        const ItemEntry e = items[2 * k + q];
        const bool has_next_item = q + 2 * (int)blockIdx.x + (k + 1) * stride < p.n_items;
        if (lane == 0) {
          if ((ok = mbar_wait(&b.q_free, (k & 1) ^ 1u, p.err))) {
            mbar_expect_tx(&b.q_full, kQBytes);
            if constexpr (PAIR) {  // tm_q has 64-row boxes here: A's queries into rows 0-63, B's into 64-127
              tma_load_2d(base, &tm_q, e.h * kD, e.w.q_row, &b.q_full);
              tma_load_2d(base + kQBytes / 2, &tm_q, (e.h2 >= 0 ? e.h2 : e.h) * kD, e.w2.q_row, &b.q_full);
            } else {
              tma_load_2d(base, &tm_q, e.h * kD, e.w.q_row, &b.q_full);
            }
          }
        }
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        const int hB = (PAIR && e.h2 >= 0) ? e.h2 : e.h;
        const __nv_bfloat16* kcol[2] = {p.pool + e.h * kD, p.pool + hB * kD};
        const __nv_bfloat16* vcol[2] = {p.pool + H + e.h * kD, p.pool + H + hB * kD};
        const bool has_b = !PAIR || e.h2 >= 0;
        for (int j = 0; j < e.n_kt; ++j, ++t) {
          const int cur[2] = {nxt[0], nxt[1]};
          if (j + 1 < e.n_kt) {
            nxt[0] = slot_of(work_of(e, 0), key_of(j + 1, 0));
            nxt[1] = slot_of(work_of(e, 1), key_of(j + 1, 1));
          } else if (has_next_item) {
            const ItemEntry& en = items[2 * (k + 1) + q];
            nxt[0] = slot_of(work_of(en, 0), key_of(0, 0));
            nxt[1] = slot_of(work_of(en, 1), key_of(0, 1));
          }
          const int st = t % kStages;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b.kv_empty[st], ((t / kStages) & 1) ^ 1u, p.err)))) break;
          const uint32_t ks = smem_u32(base + kQBytes + st * 2 * kKVBytes), vs = ks + kKVBytes;
          // eight consecutive lanes copy one key row's eight 16-byte chunks, so each copy instruction reads four whole
          // 128-byte rows; a row's slot comes from the lane that loaded it (lane R % 32 holds row R's in cur[R / 32])
          const int c = lane & 7;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int R = 4 * i + (lane >> 3);  // smem row of this lane's chunk
            const int half = i >> 3;            // R / 32
            const size_t slot = (size_t)__shfl_sync(0xffffffffu, cur[half], R & 31);
            const int key = PAIR ? j * kPairKeys + (R & 31) : j * kKTile + R;
            const bool valid = key < work_of(e, half).L && (half == 0 || has_b);
            const uint32_t off = R * 128 + ((c ^ (R & 7)) << 4);
            const uint32_t nb = valid ? 16u : 0u;
            cp_async16(ks + off, kcol[half] + slot * p.pool_ld + 8 * c, nb);
            cp_async16(vs + off, vcol[half] + slot * p.pool_ld + 8 * c, nb);
          }
          cp_async_arrive_noinc(&b.kv_full[st]);
        }
      }
    }
  } else if (warp < 4) {
    if (lane == 0) {  // MMA issuer of pipeline q: S_0, S_1, then P_t V_t followed by S_{t+2}
      const int q = warp - 2;
      PipeBars& b = bars[q];
      uint8_t* base = smem + q * kPipeBytes;
      const uint32_t preg = tmem + 192 * q;
      constexpr uint32_t idesc_qk = idesc_bf16(kQTile, kKTile);
      constexpr uint32_t idesc_pv = idesc_bf16(kQTile, kD, /*b_mn_major=*/true);
      int n_items_q = 0, total = 0;
      for (int k = 0; q + 2 * (int)blockIdx.x + k * stride < p.n_items; ++k) {
        ++n_items_q;
        total += items[2 * k + q].n_kt;
      }
      // S side cursor: item ks, tile js of it, global tile ts; P V side: item kp, tile jp, global tile tp
      int ks = 0, js = 0, ts = 0, kp = 0, jp = 0;
      bool ok = true;
      auto issue_s = [&]() -> bool {
        if (js == 0 && !mbar_wait(&b.q_full, ks & 1, p.err)) return false;
        if (!mbar_wait(&b.kv_full[ts % kStages], (ts / kStages) & 1, p.err)) return false;
        if constexpr (GATHER) fence_proxy_async_smem();  // cp.async wrote the tile through the generic proxy
        tc_fence_after();
        const uint32_t q0 = smem_u32(base), k0 = smem_u32(base + kQBytes + (ts % kStages) * 2 * kKVBytes);
        const uint32_t sbuf = preg + 64 * (ts & 1);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16(sbuf, sdesc_sw128(q0 + 32 * kk, 1024, 16), sdesc_sw128(k0 + 32 * kk, 1024, 16), idesc_qk, kk ? 1u : 0u);
        umma_commit(&b.s_full[ts & 1]);
        ++ts;
        if (++js == items[2 * ks + q].n_kt) {
          umma_commit(&b.q_free);
          js = 0;
          ++ks;
        }
        return true;
      };
      for (int i = 0; i < 2 && ts < total && ok; ++i) ok = issue_s();
      for (int tp = 0; tp < total && ok; ++tp) {
        if (!(ok = mbar_wait(&b.p_full[tp & 1], (tp >> 1) & 1, p.err))) break;
        // an item's first P V overwrites O: the softmax has read the previous item's O
        if (jp == 0 && kp > 0 && !(ok = mbar_wait(&b.o_free, (kp - 1) & 1, p.err))) break;
        tc_fence_after();
        const int st = tp % kStages;
        const uint32_t v0 = smem_u32(base + kQBytes + st * 2 * kKVBytes + kKVBytes);
        const uint32_t pbuf = preg + 64 * (tp & 1), oreg = preg + 128;
#pragma unroll
        for (int kk = 0; kk < kKTile / 16; ++kk)
          umma_f16_ts(oreg, pbuf + 8 * kk, sdesc_sw128(v0 + kk * 16 * 128, 1024, 8192), idesc_pv,
                      (jp > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&b.o_done[tp & 1]);
        umma_commit(&b.kv_empty[st]);
        if (++jp == items[2 * kp + q].n_kt) {
          jp = 0;
          ++kp;
        }
        if (ts < total) ok = issue_s();
      }
      (void)n_items_q;
    }
  } else {
    const int q = (warp - 4) >> 2;  // pipeline
    const int qw = warp & 3;        // TMEM lane quarter
    const int r = qw * 32 + lane;   // query row of the tile
    const int sub = PAIR ? (qw >> 1) : 0;  // paired form: this row's item (A: rows 0-63, B: rows 64-127)
    const int rs = r - kPairRows * sub;    // query row within its item
    PipeBars& b = bars[q];
    const uint32_t lanes = (uint32_t)(qw * 32) << 16;
    const uint32_t preg = tmem + 192 * q + lanes, oreg = preg + 128;
    int t = 0;  // global tile counter of this pipeline
    bool ok = true;
    // The previous item's output, finished during the next item's first tile: its last P V has completed by then, so
    // the O read does not wait on the tensor core (O is read before that item's first P V overwrites it: o_free).
    struct Pending {
      AttnWork w;
      int h, lim, t_last;
      float l;
    } pend;
    bool have_pend = false;
    auto finish = [&](const Pending& pd) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&b.o_done[pd.t_last & 1], (pd.t_last >> 1) & 1, p.err))) return false;
      tc_fence_after();
      float o[kD];
      tmem_ld32p(oreg, o);
      tmem_ld32p(oreg + 32, o + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b.o_free);
      const AttnWork& w = pd.w;
      const int h = pd.h, lim = pd.lim;
      const float l = pd.l;
      if (lim > 0) {
        const float inv = 1.f / l;
        const int row = w.q_row + rs;
        if constexpr (E4M3) {
          // two 32-column blocks per head, each with its own power-of-two scale
          uint8_t* dst = static_cast<uint8_t*>(p.out) + (size_t)row * p.ldo + h * kD;
          uint32_t eb[2];
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(o[32 * hb + i]));
            eb[hb] = ue8m0_for_amax(amax * inv);
            const float f = inv * ue8m0_inv(eb[hb]);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float* q = o + 32 * hb + 16 * u;
              uint4 v;
              v.x = e4m3x4(q[0] * f, q[1] * f, q[2] * f, q[3] * f);
              v.y = e4m3x4(q[4] * f, q[5] * f, q[6] * f, q[7] * f);
              v.z = e4m3x4(q[8] * f, q[9] * f, q[10] * f, q[11] * f);
              v.w = e4m3x4(q[12] * f, q[13] * f, q[14] * f, q[15] * f);
              reinterpret_cast<uint4*>(dst)[2 * hb + u] = v;
            }
          }
          *reinterpret_cast<uint16_t*>(p.out_sf + sf_offset(row, 2 * h, p.ldo)) = (uint16_t)(eb[0] | (eb[1] << 8));
        } else {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + h * kD;
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
      return true;
    };
    for (int k = 0; ok; ++k) {
      const int item = q + 2 * blockIdx.x + k * stride;
      if (item >= p.n_items) break;
      const ItemEntry& ie = items[2 * k + q];
      const AttnWork w = (PAIR && sub) ? ie.w2 : ie.w;
      const int h = (PAIR && sub) ? ie.h2 : ie.h;
      const int n_kt = ie.n_kt;
      const int pos = w.q_pos + rs;
      const int lim = (PAIR && h < 0) ? 0 : GATHER ? (pos < w.P ? w.L : 0) : (pos < w.P ? w.P : (pos < w.L ? w.L : 0));
      // A warp whose 32 query rows all lie past the item's queries (a 50-frame window fills 50 rows of the 128-row
      // tile; a sequence's last tile is partial) computes no softmax: its rows' P and O are never stored, so whatever
      // the TMEM holds there only reaches those rows' discarded outputs.  It still takes part in every barrier.
      const bool idle = __all_sync(0xffffffffu, lim == 0);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kt; ++j, ++t) {
        // warp-uniform: tcgen05.ld / st below are .sync.aligned
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b.s_full[t & 1], (t >> 1) & 1, p.err)))) break;
        if (t == 0 && q == 1) {  // offset pipeline 1 from pipeline 0 (bounded spin)
          const long long t0 = clock64();
          while (clock64() - t0 < kPipeStagger) {
          }
        }
        tc_fence_after();
        const uint32_t sbuf = preg + 64 * (t & 1);
        if (!idle) {
        bool raise;
        float m_old;
        float2 rsq[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        if constexpr (PAIR) {
          // the row's own item's 32 keys of the tile (columns 32 sub ..), P over them and zeros over the other item's
          float sv[32];
          tmem_ld32(sbuf + kPairKeys * sub, sv);
          const int kb = j * kPairKeys;
          if (!__all_sync(0xffffffffu, kb + kPairKeys <= lim)) {
#pragma unroll
            for (int i = 0; i < kPairKeys; ++i)
              if (kb + i >= lim) sv[i] = -INFINITY;
          }
          float mq[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            mq[c] = fmax3(sv[16 * c], sv[16 * c + 1], sv[16 * c + 2]);
#pragma unroll
            for (int i = 3; i < 15; i += 2) mq[c] = fmax3(mq[c], sv[16 * c + i], sv[16 * c + i + 1]);
            mq[c] = fmaxf(mq[c], sv[16 * c + 15]);
          }
          const float mx = fmaxf(mq[0], mq[1]) * p.scale_log2;
          raise = mx > m + kRescaleThreshold;
          m_old = m;
          m = raise ? mx : m;
          const float m_use = (m == -INFINITY) ? 0.f : m;
          const float2 c2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_use, -m_use);
          uint32_t u[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 a = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), c2, nm2);
            const float2 e = make_float2(exp2_approx(a.x), exp2_approx(a.y));
            rsq[i & 3] = __fadd2_rn(rsq[i & 3], e);
            const uint32_t pk = pack_bf16x2(e.x, e.y);
            u[i] = sub ? 0u : pk;
            u[16 + i] = sub ? pk : 0u;
          }
          tmem_st32(sbuf, u);
        } else {
        uint32_t sr[64];
        tmem_ld64_nowait(sbuf, sr);
        tmem_ld_wait();
        const int kb = j * kKTile;
        // keys at or past the row's limit score -inf: they add nothing to the max and 2^-inf = 0 to P (warps whose
        // rows see all 64 keys of the tile skip this)
        if (!__all_sync(0xffffffffu, kb + kKTile <= lim)) {
#pragma unroll
          for (int i = 0; i < kKTile; ++i)
            if (kb + i >= lim) sr[i] = __float_as_uint(-INFINITY);
        }
        // row max: three-input maxima in four independent chains
        float mq[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          mq[c] = fmax3(__uint_as_float(sr[16 * c]), __uint_as_float(sr[16 * c + 1]), __uint_as_float(sr[16 * c + 2]));
#pragma unroll
          for (int i = 3; i < 15; i += 2)
            mq[c] = fmax3(mq[c], __uint_as_float(sr[16 * c + i]), __uint_as_float(sr[16 * c + i + 1]));
          mq[c] = fmaxf(mq[c], __uint_as_float(sr[16 * c + 15]));
        }
        float mx = fmax3(fmaxf(mq[0], mq[1]), mq[2], mq[3]) * p.scale_log2;
        // raise the reference max only when it grows by more than the threshold (p <= 2^8 fits bf16 comfortably)
        raise = mx > m + kRescaleThreshold;
        m_old = m;
        m = raise ? mx : m;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        // P = 2^(S c - m) as bf16 pairs, written back over the scores
        const float2 c2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_use, -m_use);
        uint32_t u[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 a = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), c2, nm2);
          const float2 e = make_float2(exp2_approx(a.x), exp2_approx(a.y));
          rsq[i & 3] = __fadd2_rn(rsq[i & 3], e);
          u[i] = pack_bf16x2(e.x, e.y);
        }
        tmem_st32(sbuf, u);
        }
        // O holds P_{<j} V_{<j} relative to the old reference max: rescale it (rare) once P_{j-1} V_{j-1} is done.
        // S_t's completion implies every tensor op issued before it, so the skipped waits of o_done never fall two
        // phases behind.
        if (j > 0 && __any_sync(0xffffffffu, raise)) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&b.o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, p.err)))) break;
          tc_fence_after();
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
        const float2 rs2 = __fadd2_rn(__fadd2_rn(rsq[0], rsq[1]), __fadd2_rn(rsq[2], rsq[3]));
        l += rs2.x + rs2.y;
        tmem_st_wait();
        }
        if (j == 0 && have_pend) {  // the previous item's output (before this tile's P V can overwrite O)
          if (!(ok = finish(pend))) break;
          have_pend = false;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b.p_full[t & 1]);
      }
      if (!ok) break;
      pend.w = w;
      pend.h = h;
      pend.lim = lim;
      pend.t_last = t - 1;
      pend.l = l;
      have_pend = true;
    }
    if (ok && have_pend) finish(pend);
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool make_attn_tmaps(CUtensorMap* tm_q, CUtensorMap* tm_kv, const void* qkv, int rows, int heads) {
  const uint64_t cols = 3ull * heads * kD;
  return make_tmap_2d(tm_q, qkv, 2, (uint64_t)rows, cols, cols * 2, kQTile, kD) &&
         make_tmap_2d(tm_kv, qkv, 2, (uint64_t)rows, cols, cols * 2, kKTile, kD);
}

bool make_attn_pair_tmap(CUtensorMap* tm_q, const void* qkv, int rows, int heads) {
  const uint64_t cols = 3ull * heads * kD;
  return make_tmap_2d(tm_q, qkv, 2, (uint64_t)rows, cols, cols * 2, kPairRows, kD);
}

namespace {

template <bool E4M3, bool GATHER, bool PAIR>
int launch_attn_impl(const AttnArgs& a, cudaStream_t st, const CUtensorMap* tm_q, const CUtensorMap* tm_kv) {
  static std::atomic<uint64_t> attr_done{0};
  {
    const cudaError_t e = smem_attr_once(k_attn<E4M3, GATHER, PAIR>, kSmem, attr_done);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return T2W_ERR_CUDA;
    }
  }
  CUtensorMap mq, mkv;
  if constexpr (PAIR) {  // the query map with 64-row boxes; the gathered form reads no key map
    if (!tm_q) {
      if (!make_attn_pair_tmap(&mq, a.qkv, a.rows, a.heads)) return T2W_ERR_INVALID;
      tm_q = &mq;
    }
    tm_kv = tm_q;
  } else if (!tm_q || !tm_kv) {
    if (!make_attn_tmaps(&mq, &mkv, a.qkv, a.rows, a.heads)) return T2W_ERR_INVALID;
    tm_q = &mq;
    tm_kv = &mkv;
  }
  const int n_flat = a.n_work * a.heads;
  const int n_items = PAIR ? (n_flat + 1) / 2 : n_flat;
  DevArgs p{a.work,    n_items,  a.heads, n_flat, a.out,  a.out_sf, a.heads * kD, a.scale_log2,
            a.err,     a.pool,   a.kv_idx, a.pool_ld, a.pf, a.pf_bytes};
  int grid = (n_items + 1) / 2;
  if (grid > num_sms()) grid = num_sms();
  // each CTA stages at most kMaxCtaItems items in shared memory
  const int min_grid = (n_items + kMaxCtaItems - 1) / kMaxCtaItems;
  if (grid < min_grid) grid = min_grid;
  cudaError_t e = launch_k(k_attn<E4M3, GATHER, PAIR>, dim3(grid), dim3(384), kSmem, st, *tm_q, *tm_kv, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return T2W_OK;
}

}  // namespace

int launch_attn(const AttnArgs& a, cudaStream_t st, const CUtensorMap* tm_q, const CUtensorMap* tm_kv) {
  if (!a.qkv || !a.work || !a.out || a.rows <= 0 || a.heads <= 0 || a.n_work < 0) return T2W_ERR_INVALID;
  if (a.out_sf && (reinterpret_cast<uintptr_t>(a.out_sf) & 1)) return T2W_ERR_INVALID;
  if (a.n_work == 0) return T2W_OK;
  if (a.pool) {  // gathered keys from the slot pool (bf16 output only)
    if (a.out_sf || !a.kv_idx || a.pool_ld < 2 * a.heads * kD || a.pool_ld % 8 ||
        (reinterpret_cast<uintptr_t>(a.pool) & 15))
      return T2W_ERR_INVALID;
    if (a.pair) return launch_attn_impl<false, true, true>(a, st, a.tm_q_pair, nullptr);
    return launch_attn_impl<false, true, false>(a, st, tm_q, tm_kv);
  }
  if (a.pair) return T2W_ERR_INVALID;  // the paired form reads gathered keys only
  return a.out_sf ? launch_attn_impl<true, false, false>(a, st, tm_q, tm_kv)
                  : launch_attn_impl<false, false, false>(a, st, tm_q, tm_kv);
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
        (int64_t)seq_row[s] + seq_len[s] > rows)
      return T2W_ERR_INVALID;
    for (int q = 0; q < seq_len[s]; q += 128) work.push_back(AttnWork{seq_row[s] + q, seq_row[s], q, prompt_len[s], seq_len[s]});
  }
  if (work.size() > (size_t)kNoAllocMaxWork) return T2W_ERR_INVALID;  // beyond the fixed scratch array
  if (work.empty()) return T2W_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The work list is copied from a host vector that dies when this call returns: a capture would record a copy from
  // freed host memory, so a capturing stream is refused (nothing is enqueued and the capture stays valid).
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  if (cs != cudaStreamCaptureStatusNone) return T2W_ERR_INVALID;
  int dev = 0;
  e = cudaGetDevice(&dev);
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

// Test entry: the gathered (slot-pool) attention on host-given work and key lists, in the single or the paired form.
extern "C" int t2w_test_attn_gathered(const void* qkv, int32_t rows, int32_t heads, int32_t n_work, const int32_t* work,
                                      const void* pool, int32_t pool_rows, int32_t pool_ld, const int32_t* kv_idx,
                                      int32_t n_idx, int32_t pair, void* out, int32_t* err, void* stream) {
  using namespace t2w;
  if (!qkv || !pool || !out || !work || !kv_idx || rows <= 0 || heads <= 0 || n_work <= 0 || pool_rows <= 0 ||
      n_idx <= 0)
    return T2W_ERR_INVALID;
  std::vector<AttnWork> w(n_work);
  for (int i = 0; i < n_work; ++i) {
    w[i] = AttnWork{work[5 * i], work[5 * i + 1], work[5 * i + 2], work[5 * i + 3], work[5 * i + 4]};
    const AttnWork& x = w[i];
    const int nq = x.P - x.q_pos;  // this tile's queries
    if (x.q_row < 0 || x.q_pos < 0 || nq <= 0 || nq > (pair ? 64 : 128) || x.q_row + nq > rows || x.L <= 0 ||
        x.k_row < 0 || (int64_t)x.k_row + x.L > n_idx)
      return T2W_ERR_INVALID;
  }
  for (int j = 0; j < n_idx; ++j)
    if (kv_idx[j] < 0 || kv_idx[j] >= pool_rows) return T2W_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AttnWork* dw = nullptr;
  int* di = nullptr;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&dw), w.size() * sizeof(AttnWork));
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&di), (size_t)n_idx * 4);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dw, w.data(), w.size() * sizeof(AttnWork), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(di, kv_idx, (size_t)n_idx * 4, cudaMemcpyHostToDevice, st);
  int rc = T2W_OK;
  if (e == cudaSuccess) {
    AttnArgs a;
    a.qkv = qkv;
    a.rows = rows;
    a.heads = heads;
    a.work = dw;
    a.n_work = n_work;
    a.out = out;
    a.scale_log2 = (float)(1.4426950408889634 / 8.0);
    a.pool = static_cast<const __nv_bfloat16*>(pool);
    a.kv_idx = di;
    a.pool_ld = pool_ld;
    a.err = err;
    a.pair = pair != 0;
    rc = launch_attn(a, st);
    e = cudaStreamSynchronize(st);
  }
  cudaFree(dw);
  cudaFree(di);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return T2W_ERR_CUDA;
  }
  return rc;
}
