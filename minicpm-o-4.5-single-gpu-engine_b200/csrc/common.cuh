// Shared device helpers for the sm_100a Token2Wav kernels: mbarriers with bounded waits, TMA tile loads (no cluster
// multicast anywhere in this library), tcgen05 (UMMA) descriptors, issue, commit and TMEM access.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/t2w_b200.h"

#define T2W_DEV __device__ __forceinline__

namespace t2w {

// Every spin-wait in this library gives up after this long, records T2W_ERR_TIMEOUT in the caller's error word and
// lets the kernel run to its end (TMEM is still released), so a lost arrival never hangs the GPU.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// The same limit in SM clock cycles, for polling loops that read the cheap SM-local clock instead of %globaltimer
// (about 2 s at the B200's 1.965 GHz maximum clock; longer at lower clocks).
constexpr long long kWaitLimitCycles = 4000000000ll;

T2W_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

T2W_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
T2W_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
T2W_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
T2W_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
T2W_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
T2W_DEV bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe of a phase (for loops that poll several barriers: try_wait may suspend the thread for a while).
T2W_DEV bool mbar_test(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of parity `parity` to complete; false (and the error word set) after kWaitLimitNs.
T2W_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, T2W_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA (tiled, no multicast)
T2W_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
T2W_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completing on `bar`.
T2W_DEV void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Generic-proxy shared-memory writes made visible to the async proxy (tensor core operand reads).
T2W_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05 / TMEM
T2W_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
T2W_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
T2W_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
T2W_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
T2W_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 x bf16 -> fp32 (kind::f16), one CTA.
T2W_DEV void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A * B^T with e4m3 operands (kind::f8f6f4), fp32 accumulate.
T2W_DEV void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= (A * 2^sfA) * (B * 2^sfB)^T with e4m3 operands and UE8M0 scales per row and 32-element K block
// (kind::mxf8f6f4, one scale vector per instruction of K = 32).  The scales sit in TMEM at sfa / sfb; the byte of the
// 32-bit TMEM word that each instruction reads is the scale-factor id of `idesc`.
T2W_DEV void umma_mxf8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa_tmem,
                       uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}
// Shared memory -> TMEM copy of a 32-row x 16-byte tile, replicated into all four lane quarters (the layout of a
// scale-factor atom: row m % 32 of 128 rows in lane m % 32, byte 4 (m / 32) + k-block).
T2W_DEV void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
T2W_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major unless b_mn_major, M, N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor, kind::mxf8f6f4 with block scaling: D fp32, A/B e4m3 (format 0), K-major, UE8M0 scales
// (bit 23), scale-factor ids (the byte of the TMEM scale word) for A in bits 29-30 and for B in bits 4-5.
__host__ __device__ constexpr uint32_t idesc_mxf8(int M, int N, uint32_t sf_id) {
  return ((sf_id & 3u) << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | ((sf_id & 3u) << 29);
}
// Instruction descriptor, kind::f8f6f4: D fp32, A/B e4m3 (format 0), K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.  For K-major tiles (rows of 128 bytes) the
// stride byte offset is the 8-row group pitch (1024); for MN-major tiles it is the pitch of 8 K-rows (1024) too.
T2W_DEV uint64_t sdesc_sw128(uint32_t saddr, uint32_t sbo_bytes, uint32_t lbo_bytes) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Shared-memory matrix descriptor without swizzle (8-row x 16-byte core matrices); used for the 32 x 16-byte
// scale-factor atoms, where both strides are the 128-byte pitch of consecutive core matrices.
T2W_DEV uint64_t sdesc_noswz(uint32_t saddr, uint32_t sbo_bytes, uint32_t lbo_bytes) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// 32 lanes x 32 consecutive 32-bit columns; the wait is inside the same asm block so no use of the registers can be
// scheduled before the load has landed.
T2W_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
T2W_DEV void tmem_ld32p(uint32_t taddr, float* v) {
  float t[32];
  tmem_ld32(taddr, t);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = t[i];
}
// 32 lanes x 64 columns without waiting (the caller issues tmem_ld_wait() before using the registers).
T2W_DEV void tmem_ld64_nowait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
T2W_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
T2W_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of this library is launched with programmatic stream serialization: it may start while its predecessor
// drains.  pdl_wait() blocks until the predecessor grid has completed and its memory is visible; each kernel calls it
// before touching activations and before allocating TMEM (so an early CTA never holds TMEM its predecessor needs).
// pdl_launch() then lets the successor start launching.
T2W_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
T2W_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- launch attributes
// A kernel's MaxDynamicSharedMemorySize attribute belongs to the device it was set on: a process that drives several
// GPUs must set it on each.  `done` keeps one bit per device ordinal (devices from 64 on set it at every launch).
template <class K>
inline cudaError_t smem_attr_once(K* kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// ---------------------------------------------------------------- L2 prefetch
// Bring piece `piece` (64 KB) of [p, p + bytes) into L2: the weights of a GEMM that follows, HBM-resident (all blocks'
// weights together exceed L2) and read by every CTA of that GEMM's first round.  Each block of the issuing kernel
// takes one piece.
constexpr unsigned kPrefetchPiece = 64u << 10;
T2W_DEV void prefetch_l2_piece(const void* p, unsigned bytes, int piece) {
  const unsigned off = (unsigned)piece * kPrefetchPiece;
  if (p && off < bytes) {
    const unsigned n = bytes - off < kPrefetchPiece ? bytes - off : kPrefetchPiece;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(p) + off), "r"(n & ~15u)
                 : "memory");
  }
}

// ---------------------------------------------------------------- small math
T2W_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Packed fp32 pair arithmetic (sm_100): one instruction for two lanes of work.
T2W_DEV float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
T2W_DEV float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
T2W_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x with the hardware approximation (ex2.approx, flush-to-zero); used for softmax weights rounded to bf16 afterwards.
T2W_DEV float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
T2W_DEV float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
T2W_DEV float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanh_approx(k0 * (x + k1 * x * x * x)));
}
// Mish(y) = y tanh(softplus(y)); with e = exp(y), tanh(log(1 + e)) = e (e + 2) / (e (e + 2) + 2).  softplus is the
// identity above 20 (torch's threshold), where tanh(softplus(y)) is 1 in fp32.
T2W_DEV float mish(float y) {
  if (y > 20.f) return y;
  const float e = __expf(y);
  const float n = e * (e + 2.f);
  return y * __fdividef(n, n + 2.f);
}
// SiLU (swish) y sigmoid(y) = y / (1 + e^-y); for very negative y the exponential overflows to inf and y / inf = -0.
T2W_DEV float silu(float y) { return __fdividef(y, 1.f + __expf(-y)); }
// ---------------------------------------------------------------- cross-CTA flags (gpu scope)
T2W_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
T2W_DEV void red_release_add_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// L2 eviction priority for data a later kernel reads again (an access policy for .L2::cache_hint loads and stores;
// no device setting is changed): lines touched with it are evicted after the normal ones.
T2W_DEV uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// L2 only (.cg): the rows read this way are rewritten by other SMs between two reads (the residual stream, updated by
// GEMM epilogues and read by the norms after them), so no SM may serve them from its own L1.
T2W_DEV float4 ld_f4_l2hint(const float4* a, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(a), "l"(policy));
  return v;
}
T2W_DEV void st_f4_l2hint(float4* a, float4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(a), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w), "l"(policy)
               : "memory");
}
// Async-proxy (TMA) global writes ordered before this thread's later generic-proxy operations.
T2W_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Bounded wait until *f >= target; false (and T2W_ERR_TIMEOUT in err) after limit_ns (0: kWaitLimitNs).
T2W_DEV bool wait_counter(const int* f, int target, int* err, unsigned long long limit_ns = 0) {
  if (ld_acquire_gpu(f) >= target) return true;
  const unsigned long long limit = limit_ns ? limit_ns : kWaitLimitNs;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_gpu(f) < target) {
    __nanosleep(128);
    if (globaltimer() - t0 > limit) {
      if (err) atomicExch(err, T2W_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- e4m3 with power-of-two (UE8M0) block scales
// The UE8M0 byte e of a block whose largest magnitude is amax: the smallest power of two 2^(e - 127) with
// amax / 2^(e - 127) <= 448 (the e4m3 maximum); an all-zero block gets e = 127 (scale 1).  With amax = m 2^E,
// m in [1, 2): e - 127 = E - 8 + (m > 1.75).
T2W_DEV uint32_t ue8m0_for_amax(float amax) {
  const uint32_t u = __float_as_uint(amax);
  if (u == 0u) return 127u;
  int s = (int)(u >> 23) - 127 - 8 + ((u & 0x7fffffu) > 0x600000u ? 1 : 0);
  s = s < -127 ? -127 : (s > 127 ? 127 : s);
  return (uint32_t)(s + 127);
}
// 2^(127 - e): the factor that maps a block with scale byte e into [-448, 448] (e <= 253).
T2W_DEV float ue8m0_inv(uint32_t e) { return __uint_as_float((254u - e) << 23); }
// Two fp32 values -> two e4m3 bytes (round to nearest even, saturating): lo in bits 0-7, hi in bits 8-15.
T2W_DEV uint32_t e4m3x2(float lo, float hi) {
  unsigned short v;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(v) : "f"(hi), "f"(lo));
  return v;
}
T2W_DEV uint32_t e4m3x4(float a, float b, float c, float d) { return e4m3x2(a, b) | (e4m3x2(c, d) << 16); }
// Byte offset of (row, 32-column block j) inside the scale-factor atoms of a [rows, C] e4m3 matrix: one 512-byte atom
// per (128-row tile, 128-column block), row r of the tile at (r % 32) * 16 + (r / 32) * 4, block j at byte j % 4.
T2W_DEV uint32_t sf_offset(int row, int j, int C) {
  const int r = row & 127;
  return (uint32_t)(((row >> 7) * (C >> 7) + (j >> 2)) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (j & 3));
}

T2W_DEV uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace t2w
