// Device helpers shared by the exactkv_b200 kernels (sm_100a): inline-PTX
// wrappers for mbarriers, TMA tensor loads, bf16 mma.sync, movmatrix and ex2,
// plus the byte-parallel decoder of the compressed format.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "../../include/exactkv_b200.h"

namespace exk {

constexpr int kD = EXK_HEAD_DIM;  // head dimension (channels)
constexpr int kP = EXK_PAGE;      // tokens per page
// Bound on every spin-wait in these kernels (the mbarrier waits).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Keeps the first error: later faults do not overwrite it.
__device__ __forceinline__ void set_status(int32_t* st, int32_t code) {
  if (st != nullptr) atomicCAS(st, 0, code);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- decoding
//
// Byte-parallel rebuild of four bf16 values. Every 32-bit argument holds one
// byte per value:
//   smw  sign|mantissa bytes (sign in bit 7)
//   c    exponent codes, 0..15, one per byte (the nibble already extracted)
//   adj  base & 0x7F (the exponent base of the value's channel)
//   bb   the base byte itself (bit 7 set: the group holds zeros)
// exponent = adj + c, except that code 0 in a zero group means exponent 0
// (exactkv/codec.py:12-14, exactkv/kernels.py:96-103). No byte carries into
// its neighbour: adj + c <= 127 + 15 and c + 0x7F <= 0x8E.
// Outputs: w01 = bf16(value 0) | bf16(value 1) << 16, w23 likewise — the
// byte order of the inputs decides which values pair up (the attention
// kernel interleaves two tokens' bytes beforehand to pair along tokens).
// KILL = false is the decoder for words whose base bytes all have bit 7 clear
// (no zero group): then adj == bb and the code-0 rule cannot apply.
template <bool KILL = true>
__device__ __forceinline__ void dec4(uint32_t smw, uint32_t c, uint32_t adj, uint32_t bb,
                                     uint32_t& w01, uint32_t& w23) {
  uint32_t e = adj + c;
  if constexpr (KILL) {
    // bit 7 of each byte: code >= 1, or not a zero group; PRMT selector 8..B
    // replicates that bit over its byte, giving a 0x00/0xFF keep mask.
    const uint32_t keep = prmt((c + 0x7F7F7F7Fu) | ~bb, 0u, 0xBA98u);
    e &= keep;
  }
  const uint32_t hi = (smw & 0x80808080u) | ((e >> 1) & 0x7F7F7F7Fu);  // sign | exponent[7:1]
  const uint32_t lo = (smw & 0x7F7F7F7Fu) | ((e << 7) & 0x80808080u);  // exponent[0] | mantissa
  w01 = prmt(lo, hi, 0x5140u);
  w23 = prmt(lo, hi, 0x7362u);
}

__device__ __forceinline__ uint32_t lo_nibbles(uint32_t c) { return c & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t c) { return (c >> 4) & 0x0F0F0F0Fu; }

// dec4 on a whole code byte word: HI picks its high nibbles (channel j + 64)
// instead of the low ones (channel j); SEL0/SEL1 are the PRMT selectors that
// pair the four values into the two output words (0x5140/0x7362: values (0,1),
// (2,3); 0x6240/0x7351: (0,2), (1,3)). (Moving the shifts and additions to the
// FMA pipe as IMADs by opaque constants measured slower in the attention
// kernel: 90.8 vs 84.1 us at 32x4096.)
template <bool KILL, bool HI, uint32_t SEL0, uint32_t SEL1>
__device__ __forceinline__ void dec4f(uint32_t smw, uint32_t cw, uint32_t adj, uint32_t bb, uint32_t& w0,
                                      uint32_t& w1) {
  const uint32_t c = HI ? (cw >> 4) & 0x0F0F0F0Fu : cw & 0x0F0F0F0Fu;
  uint32_t e = adj + c;
  if constexpr (KILL) e &= prmt((c + 0x7F7F7F7Fu) | ~bb, 0u, 0xBA98u);
  const uint32_t hi = (smw & 0x80808080u) | ((e >> 1) & 0x7F7F7F7Fu);
  const uint32_t lo = (smw & 0x7F7F7F7Fu) | ((e << 7) & 0x80808080u);
  w0 = prmt(lo, hi, SEL0);
  w1 = prmt(lo, hi, SEL1);
}

// ---------------------------------------------------------------- ldmatrix

// Four 8x8 b16 matrices, transposed: lanes 8i..8i+7 give the row addresses of
// matrix i; lane (g = lane/4, t = lane%4) receives, from matrix i, the
// elements (row 2t, column g) and (row 2t+1, column g) in register i.
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& d0, uint32_t& d1, uint32_t& d2, uint32_t& d3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
               : "r"(addr));
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Adds `bytes` to the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with parity `parity` to complete; gives up
// after limit_ns (the kernels use kWaitLimitNs) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- TMA

// 3-D tiled tensor load into this CTA's shared memory, completing on `bar`.
// No multicast: every load reads this GPU's own memory for this CTA only.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Plain bulk copy of `bytes` (a multiple of 16; both addresses 16-byte
// aligned) from global to this CTA's shared memory, completing on `bar`.
// No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(static_cast<uint64_t>(__cvta_generic_to_global(src))), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------- math

// D += A * B for one m16n8k16 bf16 tile with fp32 accumulation.
// A regs: (row g, k 2t..2t+1), (row g+8, k 2t..), (row g, k 2t+8..), (row g+8, k 2t+8..)
// B regs: (k 2t..2t+1, col g), (k 2t+8..2t+9, col g);  D: (g, 2t..2t+1), (g+8, 2t..2t+1)
// with g = lane / 4, t = lane % 4.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transposes the 8x8 b16 matrix held one row per lane group (lane/4 = row,
// lane%4 = column pair) across the warp.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// 2^x with the hardware approximation (the same instruction Triton's tl.exp2
// uses); ex2(-inf) = +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace exk
