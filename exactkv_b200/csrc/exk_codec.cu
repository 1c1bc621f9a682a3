// Page encoder and decode-to-bf16 for the exponent-coded KV format (sm_100a).
//
// Encoder: one warp encodes one (sequence, page, KV head) of 16 tokens x 128
// channels. Lane (q = lane%16, th = lane/16) holds channels 4q..4q+3 and
// 64+4q..64+4q+3 of tokens 8th..8th+7, so a channel's 16 exponents live in
// lanes q and q+16 and one shuffle completes every per-channel reduction.
// Raw-pool slots are assigned in (sequence, page, head) order — the order the
// reference's encode_reference writes them (exactkv/codec.py:49-53) — by
// launches that never wait on one another: encode_kernel writes sm, code, base
// and rowmask; then for a prefill, chunk_sums / chunk_scan / chunk_place
// (below) turn the pages' raw-row counts into rowoff from the pool counter,
// advance it and copy every escaped row into its slot; for a one-token append,
// raw_offsets_kernel (one CTA) scans the page-heads and raw_copy_kernel copies.
// The reference takes a slot range with one atomic_add per page-head
// (exactkv/kernels.py:261-268), whose order depends on scheduling.
#include <algorithm>

#include "exk_device.cuh"
#include "exk_host.h"

namespace exk {

constexpr int kEncWarps = 8;
constexpr int kScanThreads = 1024;

// The kernels after the first of a call are programmatic dependents of the
// kernel before them on the stream (launch_after): they may become resident
// while it runs its last wave, which hides their launch latency, and wait in
// after_prior() until it has completed and its writes are visible (a no-op
// after an ordinary launch). allow_dependents() lets them be scheduled.
__device__ __forceinline__ void after_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() {
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

struct EncArgs {
  const uint16_t* src;
  int64_t s_b, s_pg, s_p, s_h;
  uint8_t* sm;
  uint8_t* code;
  uint8_t* base;
  int32_t* rowmask;
  int32_t* rowoff;
  uint16_t* raw;
  int64_t raw_cap;
  int32_t* cnt;
  int b0, pg0, nb, npg, H, TS, NP;
  int n_ph;
  // Append mode (one token per step, every launch enqueued once and replayed):
  // src is the tail area [B, H, 16, 128] at raw row tail_row0, T_dev the
  // tokens held before this step. encode_kernel first writes app_x[b, h] into
  // tail row T % 16; when that completes page (T + 1) / 16 - 1 the three
  // kernels encode it (pg0 comes from T_dev) and raw_copy_kernel opens the
  // next tail page; otherwise they return at once.
  // With T_stride 1 every sequence has its own length T_dev[b] (a
  // variable-length batch): each sequence appends at its own row and
  // completes its pages on its own steps.
  const int32_t* T_dev;
  int T_stride;
  const uint16_t* app_x;
  int64_t app_sb, app_sh;
  int64_t tail_row0;
};

// Tokens sequence b holds before this step (append mode).
__device__ __forceinline__ int step_length(const EncArgs& a, int b) {
  return a.T_dev[static_cast<int64_t>(b) * a.T_stride];
}

// First page of sequence b in this launch: a.pg0, or in append mode the page
// the step completes (false: the step completes no page of b).
__device__ __forceinline__ bool launch_page(const EncArgs& a, int b, int& pg0) {
  if (a.T_dev == nullptr) {
    pg0 = a.pg0;
    return true;
  }
  const int T1 = step_length(a, b) + 1;
  if (T1 % kP != 0 || T1 > a.TS) return false;
  pg0 = T1 / kP - 1;
  return true;
}

// Sequence (launch-relative) of page-head ph.
__device__ __forceinline__ int seq_of(const EncArgs& a, int ph) { return ph / (a.H * a.npg); }

// Page-head ph of a launch (ordered sequence, page, head) -> its index in the
// [B, TS/16, H] page arrays, and its source offset in elements.
__device__ __forceinline__ int64_t page_index(const EncArgs& a, int pg0, int ph, int& bi, int& pg, int& hk) {
  hk = ph % a.H;
  pg = (ph / a.H) % a.npg;
  bi = ph / (a.H * a.npg);
  return (static_cast<int64_t>(a.b0 + bi) * a.NP + pg0 + pg) * a.H + hk;
}

// Constants the compiler cannot see (2^25, 2^24, 1, 2), so that shifts and
// lane-wise adds of the encoder become multiplies on the FMA pipe: the encoder
// keeps the ALU pipe busy. A lane-wise add is a plain 32-bit add when neither
// 16-bit lane can carry into the next: the lanes then hold 0x8000 + e - b.
static __constant__ uint32_t c_fma[5] = {1u << 25, 1u << 24, 1u, 2u, 16u};

__device__ __forceinline__ uint32_t mulhi(uint32_t x, uint32_t k) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(k));
  return d;
}
__device__ __forceinline__ uint32_t mad_lo(uint32_t x, uint32_t k, uint32_t y) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(k), "r"(y));
  return d;
}

// Two 16-bit lanes per word (PTX integer SIMD; add wraps within each lane).
__device__ __forceinline__ uint32_t max_u16x2(uint32_t x, uint32_t y) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
  return d;
}
__device__ __forceinline__ uint32_t min_u16x2(uint32_t x, uint32_t y) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
  return d;
}
__device__ __forceinline__ uint32_t max_s16x2(uint32_t x, uint32_t y) {
  uint32_t d;
  asm("max.s16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
  return d;
}
__device__ __forceinline__ uint32_t add_u16x2(uint32_t x, uint32_t y) {
  uint32_t d;
  asm("add.u16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
  return d;
}

template <bool VEC>
__device__ __forceinline__ void load_row_quads(const uint16_t* p, int q, uint32_t (&v)[4]) {
  if constexpr (VEC) {
    const uint2 lo = *reinterpret_cast<const uint2*>(p + 4 * q);
    const uint2 hi = *reinterpret_cast<const uint2*>(p + 64 + 4 * q);
    v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
  } else {
    v[0] = p[4 * q] | (uint32_t(p[4 * q + 1]) << 16);
    v[1] = p[4 * q + 2] | (uint32_t(p[4 * q + 3]) << 16);
    v[2] = p[64 + 4 * q] | (uint32_t(p[64 + 4 * q + 1]) << 16);
    v[3] = p[64 + 4 * q + 2] | (uint32_t(p[64 + 4 * q + 3]) << 16);
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kEncWarps * 32, 4) encode_kernel(const __grid_constant__ EncArgs a) {
  allow_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ph = blockIdx.x * kEncWarps + warp;
  if (ph >= a.n_ph) return;  // whole warp
  if (a.app_x != nullptr) {  // append mode: this warp's (sequence, head) token first
    const int b = ph / a.H, h = ph % a.H;
    const int T = step_length(a, b);
    if (T >= a.TS) return;
    const uint2 x = reinterpret_cast<const uint2*>(a.app_x + b * a.app_sb + h * a.app_sh)[lane];
    reinterpret_cast<uint2*>(const_cast<uint16_t*>(a.src) + b * a.s_b + (T % kP) * a.s_p + h * a.s_h)[lane] = x;
    __syncwarp();  // the page's rows are read below by other lanes
  }
  int pg0;
  if (!launch_page(a, a.b0 + seq_of(a, ph), pg0)) return;
  const int q = lane & 15, th = lane >> 4;
  int bi, pg, hk;
  const int64_t page = page_index(a, pg0, ph, bi, pg, hk);

  // Two streaming passes over the lane's 8 rows (the second re-reads them from
  // L1): few registers, so four CTAs (32 warps) fit on an SM to hide latency.
  // w: bf16 pairs (4q,4q+1), (4q+2,4q+3), (64+4q, ..), (64+4q+2, ..) of one row.
  // Both passes work on two values at once in 16-bit lanes (exponents are 8
  // bits, codes and their differences fit a signed 16-bit lane).
  const uint16_t* rows = a.src + bi * a.s_b + pg * a.s_pg + static_cast<int64_t>(th * 8) * a.s_p + hk * a.s_h;
  // pass 1: per-channel maximum and minimum exponent over the 16 tokens. Each
  // lane doubled (w * 2: the sign leaves its lane, the exponent fills the
  // lane's high byte) orders the values by exponent first, so the lane-wise
  // maximum and minimum carry the extreme exponents in their high bytes.
  const uint32_t k25 = c_fma[0], k24 = c_fma[1], k1 = c_fma[2], k2 = c_fma[3], k16 = c_fma[4];
  uint32_t emax2[4], emin2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    emax2[j] = 0u;
    emin2[j] = 0xFFFFFFFFu;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t w[4];
    load_row_quads<VEC>(rows + static_cast<int64_t>(i) * a.s_p, q, w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t e2 = mad_lo(w[j], k2, 0u);
      emax2[j] = max_u16x2(emax2[j], e2);
      emin2[j] = min_u16x2(emin2[j], e2);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    emax2[j] = max_u16x2(emax2[j], __shfl_xor_sync(0xFFFFFFFFu, emax2[j], 16));
    emin2[j] = min_u16x2(emin2[j], __shfl_xor_sync(0xFFFFFFFFu, emin2[j], 16));
  }

  // per channel, two channels per word in 16-bit lanes: base b = max(emax - 15,
  // 0); zero group zm = (a zero exponent and b > 0); the base byte min(b + 128
  // zm, 255); and for pass 2 the lane biases 0x8000 - b (channels 0-63), 0x8000
  // - 16 b (channels 64-127, whose codes go to the high nibble: 16 e is added)
  // and 0x8000 - (b + zm) (b + zm <= 241: every biased sum stays in its lane)
  uint32_t byte2[4], cb2[4], czb2[4], escany = 0u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t e2 = (emax2[j] >> 8) & 0x00FF00FFu;                  // lanes: emax
    const uint32_t z2 = (emin2[j] >> 8) & 0x00FF00FFu;                  // lanes: emin
    const uint32_t b2 = max_s16x2(add_u16x2(e2, 0xFFF1FFF1u), 0u);      // max(emax - 15, 0)
    const uint32_t zm2 = (min_u16x2(z2, 0x00010001u) ^ 0x00010001u) & min_u16x2(b2, 0x00010001u);
    byte2[j] = min_u16x2(add_u16x2(b2, zm2 << 7), 0x00FF00FFu);
    cb2[j] = 0x80008000u - (j < 2 ? b2 : b2 << 4);
    czb2[j] = 0x80008000u - (b2 + zm2);
    escany |= b2 & 0xFF80FF80u;                                         // b >= 128: every row escapes
  }
  const uint32_t bw[2] = {prmt(byte2[0], byte2[1], 0x6420u), prmt(byte2[2], byte2[3], 0x6420u)};
  const bool escall = escany != 0u;

  // pass 2: codes, sign|mantissa bytes and escapes, row by row. Per value:
  // code = max(e - b, 0) (a zero of a zero group gets 0); it escapes when
  // e != 0 and e < b + zm, or when b >= 128.
  uint32_t escw = escall ? 0x00FF00FFu : 0u;  // bit i / 16 + i: row i escapes in the low / high lane
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int tok = th * 8 + i;
    const int64_t row = (static_cast<int64_t>(a.b0 + bi) * a.TS + (pg0 + pg) * kP + tok) * a.H + hk;
    uint32_t w[4];
    load_row_quads<VEC>(rows + static_cast<int64_t>(i) * a.s_p, q, w);
    uint32_t code2[4], x[4], escacc = 0u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t e2 = mulhi(w[j], k25) & 0x00FF00FFu;  // (w >> 7): exponents in the low byte of each lane
      // lanes 0x8000 + max(e - b, 0) (x 16 for channels 64-127): the code in the low byte
      code2[j] = max_u16x2(mad_lo(e2, j < 2 ? k1 : k16, cb2[j]), 0x80008000u);
      // lane bit 15 of e2 + 0x8000 - (b + zm): e >= b + zm; of e2 + 0x7FFF: e != 0
      escacc |= ~mad_lo(e2, k1, czb2[j]) & mad_lo(e2, k1, 0x7FFF7FFFu);
      // bit 7 of each lane's low byte from the sign (w >> 8), bits 0-6 the
      // mantissa; the high bytes are not used
      x[j] = (mulhi(w[j], k24) & 0x00800080u) | (w[j] & 0xFF7FFF7Fu);
    }
    const uint32_t smw0 = prmt(x[0], x[1], 0x6420u), smw1 = prmt(x[2], x[3], 0x6420u);
    const uint32_t cw = prmt(code2[0] | code2[2], code2[1] | code2[3], 0x6420u);
    *reinterpret_cast<uint32_t*>(a.sm + row * kD + 4 * q) = smw0;
    *reinterpret_cast<uint32_t*>(a.sm + row * kD + 64 + 4 * q) = smw1;
    *reinterpret_cast<uint32_t*>(a.code + row * (kD / 2) + 4 * q) = cw;
    escw |= (escacc >> (15 - i)) & (0x00010001u << i);
  }
  if (th == 0) {
    *reinterpret_cast<uint32_t*>(a.base + page * kD + 4 * q) = bw[0];
    *reinterpret_cast<uint32_t*>(a.base + page * kD + 64 + 4 * q) = bw[1];
  }
  // rowmask: token 8th+i escapes if any of its 16 lanes saw an escape (bit i
  // of escrow in lanes 16th..16th+15: bit 8th+i of one warp-wide OR)
  const uint32_t escrow = (escw | (escw >> 16)) & 0xFFu;
  const uint32_t rm = __reduce_or_sync(0xFFFFFFFFu, escrow << (8 * th));
  if (lane == 0) a.rowmask[page] = static_cast<int32_t>(rm);
}

// One CTA: exclusive prefix of the launch's per-page raw-row counts, starting
// at the pool counter, in tiles of 4 page-heads per thread.
__global__ void __launch_bounds__(kScanThreads) raw_offsets_kernel(const __grid_constant__ EncArgs a) {
  __shared__ int s_warp[kScanThreads / 32];
  __shared__ int s_total;
  allow_dependents();
  after_prior();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int pg0 = a.pg0;
  if (a.T_stride == 0 && !launch_page(a, 0, pg0)) return;  // one length: uniform over the CTA
  int carry = *a.cnt;
  for (int tile = 0; tile < a.n_ph; tile += 4 * kScanThreads) {
    int cnt[4];
    int64_t idx[4];
    int local = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ph = tile + 4 * threadIdx.x + j;
      cnt[j] = 0;
      idx[j] = -1;
      int pgj;
      if (ph < a.n_ph && launch_page(a, a.b0 + seq_of(a, ph), pgj)) {  // sequences completing a page only
        int bi, pg, hk;
        idx[j] = page_index(a, pgj, ph, bi, pg, hk);
        cnt[j] = __popc(static_cast<uint32_t>(a.rowmask[idx[j]]) & 0xFFFFu);
      }
      local += cnt[j];
    }
    int incl = local;  // inclusive scan within the warp
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
      int wi = w;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, wi, d);
        if (lane >= d) wi += y;
      }
      s_warp[lane] = wi - w;  // exclusive per warp
      if (lane == 31) s_total = wi;
    }
    __syncthreads();
    int off = carry + s_warp[warp] + incl - local;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (idx[j] >= 0) a.rowoff[idx[j]] = off;
      off += cnt[j];
    }
    carry += s_total;
    __syncthreads();  // s_warp / s_total are rewritten by the next tile
  }
  if (threadIdx.x == 0) *a.cnt = carry;  // may exceed raw_cap: the caller grows the pool
}

// One warp per page-head with raw rows: copies each escaped row from the
// source into pool row rowoff + rank; rows at or past raw_cap are skipped.
template <bool VEC>
__global__ void __launch_bounds__(kEncWarps * 32) raw_copy_kernel(const __grid_constant__ EncArgs a) {
  after_prior();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ph = blockIdx.x * kEncWarps + warp;
  if (ph >= a.n_ph) return;
  int pg0;
  if (!launch_page(a, a.b0 + seq_of(a, ph), pg0)) return;
  int bi, pg, hk;
  const int64_t page = page_index(a, pg0, ph, bi, pg, hk);
  if (a.app_x != nullptr && pg0 + 1 < a.NP) {
    // open the next tail page: all its rows are raw, in this (sequence, head)'s tail rows
    const int64_t nxt = page + a.H;
    if (lane == 0) {
      a.rowmask[nxt] = 0xFFFF;
      a.rowoff[nxt] = static_cast<int32_t>(a.tail_row0 + static_cast<int64_t>(ph) * kP);
    }
  }
  uint32_t rm = static_cast<uint32_t>(a.rowmask[page]) & 0xFFFFu;
  if (rm == 0u) return;
  const int64_t ro = a.rowoff[page];
  int rank = 0;
  while (rm != 0u) {
    const int tok = __ffs(rm) - 1;
    rm &= rm - 1u;
    const int64_t ridx = ro + rank++;
    if (ridx < 0 || ridx >= a.raw_cap) continue;
    const uint16_t* s = a.src + bi * a.s_b + pg * a.s_pg + static_cast<int64_t>(tok) * a.s_p + hk * a.s_h;
    uint16_t* d = a.raw + ridx * kD;
    if constexpr (VEC) {
      reinterpret_cast<uint2*>(d)[lane] = reinterpret_cast<const uint2*>(s)[lane];
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) d[4 * lane + j] = s[4 * lane + j];
    }
  }
}

// Prefill launches (no device length) place raw rows in chunks of kChunkPh
// page-heads instead of one CTA walking them all: chunk_sums_kernel writes each
// chunk's raw-row count into the rowoff slot of the chunk's first page-head
// (free until the final offsets: every rowoff of the launch is rewritten
// below), chunk_scan_kernel (one CTA) turns those counts into offsets from the
// pool counter and advances it, and chunk_place_kernel gives every page-head of
// a chunk its offset and copies the chunk's raw rows. Same slots, same
// (sequence, page, head) order as raw_offsets_kernel + raw_copy_kernel.
constexpr int kChunkPh = 256;
constexpr int kChunkThreads = 256;  // one page-head per thread
constexpr int kCopyBatch = 8;       // raw rows a placement warp loads before storing them

__device__ __forceinline__ int64_t prefill_page(const EncArgs& a, int ph) {
  int bi, pg, hk;
  return page_index(a, a.pg0, ph, bi, pg, hk);
}

__global__ void __launch_bounds__(kChunkThreads) chunk_sums_kernel(const __grid_constant__ EncArgs a) {
  __shared__ int s_warp[kChunkThreads / 32];
  allow_dependents();
  after_prior();
  const int c0 = blockIdx.x * kChunkPh;
  int n = 0;
#pragma unroll
  for (int j = 0; j < kChunkPh / kChunkThreads; ++j) {
    const int ph = c0 + j * kChunkThreads + threadIdx.x;
    if (ph < a.n_ph) n += __popc(static_cast<uint32_t>(a.rowmask[prefill_page(a, ph)]) & 0xFFFFu);
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) n += __shfl_xor_sync(0xFFFFFFFFu, n, d);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kChunkThreads / 32; ++w) t += s_warp[w];
    a.rowoff[prefill_page(a, c0)] = t;
  }
}

__global__ void __launch_bounds__(kScanThreads) chunk_scan_kernel(const __grid_constant__ EncArgs a) {
  __shared__ int s_warp[kScanThreads / 32];
  __shared__ int s_total;
  allow_dependents();
  after_prior();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_chunks = (a.n_ph + kChunkPh - 1) / kChunkPh;
  int carry = *a.cnt;
  for (int tile = 0; tile < n_chunks; tile += kScanThreads) {
    const int c = tile + threadIdx.x;
    const int64_t idx = c < n_chunks ? prefill_page(a, c * kChunkPh) : -1;
    const int local = idx >= 0 ? a.rowoff[idx] : 0;
    int incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int w = s_warp[lane];
      int wi = w;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, wi, d);
        if (lane >= d) wi += y;
      }
      s_warp[lane] = wi - w;
      if (lane == 31) s_total = wi;
    }
    __syncthreads();
    if (idx >= 0) a.rowoff[idx] = carry + s_warp[warp] + incl - local;
    carry += s_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *a.cnt = carry;  // may exceed raw_cap: the caller grows the pool
}

template <bool VEC>
__global__ void __launch_bounds__(kChunkThreads) chunk_place_kernel(const __grid_constant__ EncArgs a) {
  __shared__ int s_off[kChunkPh];
  __shared__ uint32_t s_rm[kChunkPh];
  __shared__ int s_warp[kChunkThreads / 32];
  __shared__ int s_base;
  after_prior();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * kChunkPh;
  constexpr int kPer = kChunkPh / kChunkThreads;
  if (threadIdx.x == 0) s_base = a.rowoff[prefill_page(a, c0)];  // the chunk's offset, from chunk_scan_kernel
  // counts of this thread's kPer consecutive page-heads
  uint32_t rm[kPer];
  int local = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int ph = c0 + threadIdx.x * kPer + j;
    rm[j] = ph < a.n_ph ? static_cast<uint32_t>(a.rowmask[prefill_page(a, ph)]) & 0xFFFFu : 0u;
    local += __popc(rm[j]);
  }
  int incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int wpre = 0;
  for (int w = 0; w < warp; ++w) wpre += s_warp[w];
  int off = s_base + wpre + incl - local;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x * kPer + j;
    s_off[i] = off;
    s_rm[i] = rm[j];
    const int ph = c0 + i;
    if (ph < a.n_ph) a.rowoff[prefill_page(a, ph)] = off;
    off += __popc(rm[j]);
  }
  __syncthreads();
  // each warp copies the raw rows of its share of the chunk. The sources are
  // cold (the encode pass read them long ago), so the warp queues up to
  // kCopyBatch rows — across page-heads — and loads them all before storing.
  __shared__ int64_t s_src[kChunkThreads / 32][kCopyBatch];
  __shared__ int64_t s_dst[kChunkThreads / 32][kCopyBatch];
  int n = 0;
  auto flush = [&]() {
    __syncwarp();
    uint32_t v[kCopyBatch][2];
#pragma unroll
    for (int j = 0; j < kCopyBatch; ++j) {
      v[j][0] = v[j][1] = 0u;
      if (j < n) {
        const uint16_t* src = a.src + s_src[warp][j];
        if constexpr (VEC) {
          const uint2 x = reinterpret_cast<const uint2*>(src)[lane];
          v[j][0] = x.x;
          v[j][1] = x.y;
        } else {
          v[j][0] = src[4 * lane] | (uint32_t(src[4 * lane + 1]) << 16);
          v[j][1] = src[4 * lane + 2] | (uint32_t(src[4 * lane + 3]) << 16);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kCopyBatch; ++j) {
      if (j < n) {
        uint16_t* d = a.raw + s_dst[warp][j] * kD;
        if constexpr (VEC) {
          reinterpret_cast<uint2*>(d)[lane] = make_uint2(v[j][0], v[j][1]);
        } else {
          d[4 * lane] = static_cast<uint16_t>(v[j][0]);
          d[4 * lane + 1] = static_cast<uint16_t>(v[j][0] >> 16);
          d[4 * lane + 2] = static_cast<uint16_t>(v[j][1]);
          d[4 * lane + 3] = static_cast<uint16_t>(v[j][1] >> 16);
        }
      }
    }
    __syncwarp();
    n = 0;
  };
  for (int i = warp; i < kChunkPh; i += kChunkThreads / 32) {
    uint32_t m = s_rm[i];
    if (m == 0u) continue;
    const int ph = c0 + i;
    int bi, pg, hk;
    page_index(a, a.pg0, ph, bi, pg, hk);
    const int64_t src0 = bi * a.s_b + pg * a.s_pg + hk * a.s_h;
    int64_t ridx = s_off[i];
    while (m != 0u) {
      const int tok = __ffs(m) - 1;
      m &= m - 1u;
      if (ridx >= 0 && ridx < a.raw_cap) {
        if (lane == 0) {
          s_src[warp][n] = src0 + static_cast<int64_t>(tok) * a.s_p;
          s_dst[warp][n] = ridx;
        }
        if (++n == kCopyBatch) flush();
      }
      ++ridx;
    }
  }
  if (n > 0) flush();
}

struct DecArgs {
  const uint8_t* sm;
  const uint8_t* code;
  const uint8_t* base;
  const int32_t* rowmask;
  const int32_t* rowoff;
  const uint16_t* raw;
  int64_t raw_rows;
  uint16_t* out;
  int32_t* status;
  int B, TS, NP, H, T, NPT;
  int64_t n_ph;
};

// One warp per (sequence, page, head) of the first T tokens; same lane layout
// as the encoder and the same dec4 rebuild as the attention kernel.
__global__ void __launch_bounds__(256) decode_kernel(const __grid_constant__ DecArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ph = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (ph >= a.n_ph) return;
  const int hk = static_cast<int>(ph % a.H);
  const int pg = static_cast<int>((ph / a.H) % a.NPT);
  const int b = static_cast<int>(ph / (static_cast<int64_t>(a.H) * a.NPT));
  const int q = lane & 15, th = lane >> 4;
  const int64_t page = (static_cast<int64_t>(b) * a.NP + pg) * a.H + hk;
  const uint32_t rm = static_cast<uint32_t>(a.rowmask[page]) & 0xFFFFu;
  const int32_t ro = a.rowoff[page];
  const uint32_t bl = *reinterpret_cast<const uint32_t*>(a.base + page * kD + 4 * q);
  const uint32_t bh = *reinterpret_cast<const uint32_t*>(a.base + page * kD + 64 + 4 * q);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int tok = th * 8 + i;
    const int t_abs = pg * kP + tok;
    if (t_abs >= a.T) break;
    const int64_t row = (static_cast<int64_t>(b) * a.TS + t_abs) * a.H + hk;
    uint32_t w0, w1, w2, w3;
    if ((rm >> tok) & 1u) {
      const int64_t ridx = static_cast<int64_t>(ro) + __popc(rm & ((1u << tok) - 1u));
      if (ridx < 0 || ridx >= a.raw_rows) {
        set_status(a.status, EXK_S_RAW_INDEX);
        w0 = w1 = w2 = w3 = 0u;
      } else {
        const uint16_t* r = a.raw + ridx * kD;
        const uint2 lo = *reinterpret_cast<const uint2*>(r + 4 * q);
        const uint2 hi = *reinterpret_cast<const uint2*>(r + 64 + 4 * q);
        w0 = lo.x; w1 = lo.y; w2 = hi.x; w3 = hi.y;
      }
    } else {
      const uint32_t sl = *reinterpret_cast<const uint32_t*>(a.sm + row * kD + 4 * q);
      const uint32_t sh = *reinterpret_cast<const uint32_t*>(a.sm + row * kD + 64 + 4 * q);
      const uint32_t cw = *reinterpret_cast<const uint32_t*>(a.code + row * (kD / 2) + 4 * q);
      dec4(sl, lo_nibbles(cw), bl & 0x7F7F7F7Fu, bl, w0, w1);
      dec4(sh, hi_nibbles(cw), bh & 0x7F7F7F7Fu, bh, w2, w3);
    }
    uint16_t* o = a.out + ((static_cast<int64_t>(b) * a.T + t_abs) * a.H + hk) * kD;
    *reinterpret_cast<uint2*>(o + 4 * q) = make_uint2(w0, w1);
    *reinterpret_cast<uint2*>(o + 64 + 4 * q) = make_uint2(w2, w3);
  }
}

}  // namespace exk

using namespace exk;

namespace {

// Launches kern as a programmatic dependent of the kernel before it on the stream.
int launch_after(void (*kern)(EncArgs), int grid, int block, cudaStream_t st, const EncArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e == cudaSuccess) return 0;
  (void)cudaGetLastError();  // reported here, not by the next launch's check
  return static_cast<int>(e);
}

}  // namespace

extern "C" int exk_encode_pages(const uint16_t* src, int64_t s_b, int64_t s_pg, int64_t s_p, int64_t s_h,
                                uint8_t* sm, uint8_t* code, uint8_t* base, int32_t* rowmask, int32_t* rowoff,
                                uint16_t* raw, int64_t raw_cap, int32_t* cnt, int b0, int pg0, int nb, int npg, int H,
                                int TS, int32_t* status, int device, void* stream) {
  (void)status;  // the encoder has no waits and no metadata-driven reads to report
  if (src == nullptr || sm == nullptr || code == nullptr || base == nullptr || rowmask == nullptr ||
      rowoff == nullptr || raw == nullptr || cnt == nullptr)
    return EXK_EARG;
  if (nb <= 0 || npg <= 0 || H <= 0 || TS <= 0 || TS % kP != 0 || b0 < 0 || pg0 < 0 || raw_cap < 0) return EXK_EARG;
  if ((pg0 + npg) * kP > TS) return EXK_EARG;
  const int64_t n_ph = static_cast<int64_t>(nb) * npg * H;
  if (n_ph > (int64_t{1} << 30)) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(raw) & 7u) != 0) return EXK_EALIGN;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  EncArgs a;
  a.src = src;
  a.s_b = s_b;
  a.s_pg = s_pg;
  a.s_p = s_p;
  a.s_h = s_h;
  a.sm = sm;
  a.code = code;
  a.base = base;
  a.rowmask = rowmask;
  a.rowoff = rowoff;
  a.raw = raw;
  a.raw_cap = raw_cap;
  a.cnt = cnt;
  a.b0 = b0;
  a.pg0 = pg0;
  a.nb = nb;
  a.npg = npg;
  a.H = H;
  a.TS = TS;
  a.NP = TS / kP;
  a.n_ph = static_cast<int>(n_ph);
  a.T_dev = nullptr;
  a.T_stride = 0;
  a.app_x = nullptr;
  a.app_sb = a.app_sh = 0;
  a.tail_row0 = -1;
  const int blocks = static_cast<int>((n_ph + kEncWarps - 1) / kEncWarps);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 8-byte vector loads need every (sequence, page, token, head) start 8-byte aligned
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 7u) == 0 && (s_b % 4) == 0 && (s_pg % 4) == 0 &&
                   (s_p % 4) == 0 && (s_h % 4) == 0;
  if (vec)
    encode_kernel<true><<<blocks, kEncWarps * 32, 0, st>>>(a);
  else
    encode_kernel<false><<<blocks, kEncWarps * 32, 0, st>>>(a);
  if ((r = launch_status()) != 0) return r;
  const int chunks = static_cast<int>((n_ph + kChunkPh - 1) / kChunkPh);
  if ((r = launch_after(chunk_sums_kernel, chunks, kChunkThreads, st, a)) != 0) return r;
  if ((r = launch_after(chunk_scan_kernel, 1, kScanThreads, st, a)) != 0) return r;
  return launch_after(vec ? chunk_place_kernel<true> : chunk_place_kernel<false>, chunks, kChunkThreads, st, a);
}

extern "C" int exk_decode_to_bf16(const exk_cview* c, int B, int TS, int H, int T, uint16_t* out, int32_t* status,
                                  int device, void* stream) {
  if (c == nullptr || out == nullptr) return EXK_EARG;
  if (B <= 0 || H <= 0 || T <= 0 || TS % kP != 0 || T > TS || c->raw_rows < 0) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0 || !aligned16(c->raw) || !aligned16(c->sm) ||
      !aligned16(c->code) || !aligned16(c->base))
    return EXK_EALIGN;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  DecArgs a;
  a.sm = c->sm;
  a.code = c->code;
  a.base = c->base;
  a.rowmask = c->rowmask;
  a.rowoff = c->rowoff;
  a.raw = c->raw;
  a.raw_rows = c->raw_rows;
  a.out = out;
  a.status = status;
  a.B = B;
  a.TS = TS;
  a.NP = TS / kP;
  a.H = H;
  a.T = T;
  a.NPT = (T + kP - 1) / kP;
  a.n_ph = static_cast<int64_t>(B) * a.NPT * H;
  const int64_t blocks = (a.n_ph + 7) / 8;
  if (blocks > (int64_t{1} << 31) - 1) return EXK_EARG;
  decode_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

extern "C" int exk_append_token(const uint16_t* x, int64_t x_sb, int64_t x_sh, uint8_t* sm, uint8_t* code,
                                uint8_t* base, int32_t* rowmask, int32_t* rowoff, uint16_t* raw, int64_t raw_cap,
                                int32_t* cnt, int B, int H, int TS, const int32_t* T_dev, int T_stride,
                                int32_t* status, int device, void* stream) {
  (void)status;
  if (x == nullptr || sm == nullptr || code == nullptr || base == nullptr || rowmask == nullptr ||
      rowoff == nullptr || raw == nullptr || cnt == nullptr || T_dev == nullptr || (T_stride != 0 && T_stride != 1))
    return EXK_EARG;
  if (B <= 0 || H <= 0 || TS <= 0 || TS % kP != 0 || raw_cap < 0) return EXK_EARG;
  if (static_cast<int64_t>(B) * H > (int64_t{1} << 30)) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(x) & 7u) != 0 || (x_sb % 4) != 0 || (x_sh % 4) != 0 ||
      (reinterpret_cast<uintptr_t>(raw) & 7u) != 0 || (reinterpret_cast<uintptr_t>(T_dev) & 3u) != 0)
    return EXK_EALIGN;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  EncArgs a;
  a.src = raw + raw_cap * kD;  // the tail area [B, H, 16, 128]
  a.s_b = static_cast<int64_t>(H) * kP * kD;
  a.s_pg = 0;
  a.s_p = kD;
  a.s_h = static_cast<int64_t>(kP) * kD;
  a.sm = sm;
  a.code = code;
  a.base = base;
  a.rowmask = rowmask;
  a.rowoff = rowoff;
  a.raw = raw;
  a.raw_cap = raw_cap;
  a.cnt = cnt;
  a.b0 = 0;
  a.pg0 = 0;
  a.nb = B;
  a.npg = 1;
  a.H = H;
  a.TS = TS;
  a.NP = TS / kP;
  a.n_ph = B * H;
  a.T_dev = T_dev;
  a.T_stride = T_stride;
  a.app_x = x;
  a.app_sb = x_sb;
  a.app_sh = x_sh;
  a.tail_row0 = raw_cap;
  const int blocks = (a.n_ph + kEncWarps - 1) / kEncWarps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  encode_kernel<true><<<blocks, kEncWarps * 32, 0, st>>>(a);
  if ((r = launch_status()) != 0) return r;
  if ((r = launch_after(raw_offsets_kernel, 1, kScanThreads, st, a)) != 0) return r;
  return launch_after(raw_copy_kernel<true>, blocks, kEncWarps * 32, st, a);
}

__global__ void advance_kernel(int32_t* T_dev, int n) { *T_dev += n; }

// Copy from mapped pinned host memory by the SMs: 16-byte loads over PCIe,
// kCopyIn per thread issued before any store, so a step's few hundred KB of
// inputs cross in about one round trip.
constexpr int kCopyIn = 4;

__global__ void __launch_bounds__(256) copy_in_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * 256;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i0 < n; i0 += kCopyIn * stride) {
    uint4 v[kCopyIn];
#pragma unroll
    for (int j = 0; j < kCopyIn; ++j)
      if (i0 + j * stride < n) v[j] = src[i0 + j * stride];
#pragma unroll
    for (int j = 0; j < kCopyIn; ++j)
      if (i0 + j * stride < n) dst[i0 + j * stride] = v[j];
  }
}

extern "C" int exk_copy_from_host(void* dst, const void* src, int64_t bytes, int device, void* stream) {
  if (dst == nullptr || src == nullptr || bytes <= 0) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) != 0 ||
      bytes % 16 != 0)
    return EXK_EALIGN;
  int sms = 0;
  int r = use_device(device, &sms);
  if (r != 0) return r;
  if (device_reachable(src) != 0 || device_reachable(dst) != 0) return EXK_EARG;
  const int64_t n = bytes / 16;
  const int64_t grid = std::min<int64_t>((n + 255) / 256, 4 * static_cast<int64_t>(sms));
  copy_in_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(dst), static_cast<const uint4*>(src), n);
  return launch_status();
}

extern "C" int exk_advance_length(int32_t* T_dev, int n, int device, void* stream) {
  if (T_dev == nullptr) return EXK_EARG;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(T_dev, n);
  return launch_status();
}

// Self-test of the bounded wait every kernel uses: one thread waits on an
// mbarrier that nothing arrives at, gives up after limit_ns and records
// EXK_S_FULL_TIMEOUT, exactly as a consumer whose stage never lands would.
// No copy is in flight, so giving up is safe.
__global__ void wait_timeout_selftest(int32_t* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  if (!mbar_wait(&bar, 0u, limit_ns)) set_status(status, EXK_S_FULL_TIMEOUT);
}

extern "C" int exk_selftest_wait_timeout(int32_t* status, uint64_t limit_ns, int device, void* stream) {
  if (status == nullptr || limit_ns == 0 || limit_ns > kWaitLimitNs) return EXK_EARG;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  wait_timeout_selftest<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns);
  return launch_status();
}
