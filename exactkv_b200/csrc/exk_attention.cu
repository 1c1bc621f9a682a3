// Split-K decode attention over the exponent-coded bf16 KV cache (sm_100a),
// its uncompressed bf16 sibling, and the split merge.
//
// Work decomposition. A work item is one (sequence b, group of HG KV heads,
// token split) of the plan; persistent CTAs (one per SM) take items
// round-robin. The HG heads of a page range are one contiguous region of each
// cache buffer ([B, TS, H, *] layout), so one producer warp streams a stage =
// WPH consecutive 16-token pages of all HG heads with one TMA box per field
// (cp.async.bulk.tensor, 128B/64B swizzle, no multicast) into a ring of
// mbarrier-guarded stages. The NWC = HG x WPH consumer warps are (head, page
// phase) pairs: every warp consumes every stage, rebuilding its head's K and V
// of its page in registers straight into bf16 mma fragments and running the
// online softmax; with WPH > 1 the page phases of a head are merged through
// shared memory at the end of the item, in fixed order.
//
// Tensor-core mapping ("swapped" GQA): per 16-token page the warp computes
//   S^T[16 tok x 8 heads]  = K[16 x 128] . Q^T[128 x 8]     (8 mma, k = channels)
//   O^T[128 ch x 8 heads] += V^T[128 x 16] . P^T[16 x 8]    (8 mma, k = tokens)
// so the G query heads that share a KV head sit in the n=8 dimension (two
// n-tiles for 9 <= G <= 16) and each K/V element is read once for all of them
// (the reference packs heads into M, exactkv/kernels.py:4-8, 62-68).
//
// Bit-identity. The compressed and bf16 kernels instantiate the same template
// and differ only in how a lane fills its fragment registers; the registers
// hold the same bf16 bits in the same slots, so every mma, softmax step and
// merge runs identically (the property exactkv/kernels.py:10-18 relies on).
#include <algorithm>
#include <cfloat>
#include <cuda.h>

#include "exk_device.cuh"
#include "exk_host.h"

namespace exk {

constexpr int kRawArea = 16;              // raw rows staged per stage (compressed kernel)
constexpr int kAccPitch = 132;            // floats per head row of the merge buffer (bank padding)
constexpr uint32_t kSigma = 0x27146350u;  // mma row r (0..7) -> page token sigma(r), nibble r

// Token of the page that mma row r (0..15) holds. The permutation spreads the
// rows a quarter/half warp reads over distinct 16-byte bank groups of the
// swizzled tiles (rows r, r+1 differ in bits 0 and 2; rows 2i cover every
// value of bits 1-2).
__device__ __forceinline__ int sigma(int r) { return ((kSigma >> (4 * (r & 7))) & 0xF) | (r & 8); }

struct AttnArgs {
  const uint16_t* q;            // [B, Hq, 128]
  const int32_t* rowmask[2];    // K, V (compressed kernel only)
  const int32_t* rowoff[2];
  const uint16_t* raw[2];
  int64_t raw_rows[2];
  float* ws_o;
  float* ws_m;
  float* ws_l;
  int32_t* status;
  int B, TS, NP, Hkv, Hq, G, T;
  const int32_t* T_dev;         // if set, sequence b's valid length is T_dev[b * T_stride] + T_add
  int T_add, T_stride;          // (T is then the capacity; T_stride 0: one length for the batch)
  int ns, split_len, s0, nsl, n_items, ngroups;
  // Balanced partition (bal_G > 0): the bal_W = units x bal_Su stages of the
  // launch (a unit = one sequence's head group, bal_Su stages of WPH pages
  // each) are cut into bal_G equal runs, one per CTA (the grid is bal_G); the
  // j-th piece of CTA c's run inside one unit is item c + j * bal_G, and it is
  // split number c - (first CTA touching the unit) of that unit.
  int bal_G, bal_Su;
  int64_t bal_W;
  float qk_scale;
  // Paged caches: page pg of sequence b is page pages[b * pages_stride + pg] of
  // a pool of pool_pages pages (the cache buffers seen as [pool_pages, 16, H,
  // *]); nullptr: page b * NP + pg of the [B, TS] buffers.
  const int32_t* pages;
  int pages_stride, pool_pages;
};

// Compressed: ksm, kcode, kbase, vsm, vcode, vbase.  bf16: k, v.
struct alignas(64) AttnMaps {
  CUtensorMap m[6];
};

// Heads per CTA for a KV head count: the largest power of two <= 8 dividing it.
__host__ __device__ constexpr int head_group(int hkv) {
  return hkv % 8 == 0 ? 8 : hkv % 4 == 0 ? 4 : hkv % 2 == 0 ? 2 : 1;
}

template <bool COMP, int NT, int NWC, int HG>
struct Cfg {
  static_assert(NWC % HG == 0, "heads per CTA must divide the consumer warps");
  static constexpr int kWph = NWC / HG;                       // page phases per head
  static constexpr int kTile = COMP ? 6400 : 8192;           // one head x one page, K and V
  static constexpr int kStageBytes = NWC * kTile;
  static constexpr int kHeads = 8 * NT;                      // query heads per warp (padded)
  static constexpr int kMergeBytes = kWph > 1 ? HG * kHeads * kAccPitch * 4 : 0;
  static constexpr int kMLBytes = 2 * NWC * kHeads * 4;
  static constexpr int kMetaSlot = COMP ? NWC * 16 : 0;       // per stage: (rowmask, rowoff) x (K, V) per tile
  static constexpr int kRawRows = COMP ? kRawArea : 0;        // raw rows staged per stage
  static constexpr int kRawSlot = kRawRows * kD * 2;
  static constexpr int kBudget = 224 * 1024 - kMergeBytes - kMLBytes - 4 * (kMetaSlot + kRawSlot) - 1024;
  static constexpr int kStages = (kBudget / kStageBytes) > 4 ? 4 : (kBudget / kStageBytes);
  static_assert(kStages >= 2, "shared memory too small for two stages");
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kBarBytes = 2 * kStages * 8 + 16;
  static constexpr int kBytes =
      kRingBytes + kStages * kRawSlot + kMergeBytes + kMLBytes + kStages * kMetaSlot + kBarBytes + 1024;
  static constexpr uint32_t kTxBytes = static_cast<uint32_t>(kStageBytes);
};

// Shared-memory layout of one stage. Compressed: sm [K,V][HG][16*WPH rows][128 B]
// (128B swizzle), code [K,V][HG][16*WPH][64 B] (64B swizzle), base [K,V][HG][WPH][128 B].
// bf16: [K lo, K hi, V lo, V hi][HG][16*WPH][128 B] (128B swizzle; lo = channels 0-63).
// The tile of (head h, page phase ph) starts at a 1024-byte multiple, so the
// swizzle phase of its row r is r & 7 whatever h and ph are.
struct Slot {
  const uint8_t* p[6];
};

template <bool COMP, int NWC, int HG>
__device__ __forceinline__ Slot tile_ptrs(const uint8_t* stage, int h, int ph) {
  constexpr int WPH = NWC / HG;
  const int u = h * WPH + ph;  // tile index within a field
  Slot o;
  if constexpr (COMP) {
    const uint8_t* sm = stage;
    const uint8_t* cd = stage + NWC * 4096;
    const uint8_t* bs = stage + NWC * 6144;
    o.p[0] = sm + u * 2048;
    o.p[1] = cd + u * 1024;
    o.p[2] = bs + u * 128;
    o.p[3] = sm + NWC * 2048 + u * 2048;
    o.p[4] = cd + NWC * 1024 + u * 1024;
    o.p[5] = bs + NWC * 128 + u * 128;
  } else {
    o.p[0] = stage + u * 2048;
    o.p[1] = stage + NWC * 2048 + u * 2048;
    o.p[2] = stage + 2 * NWC * 2048 + u * 2048;
    o.p[3] = stage + 3 * NWC * 2048 + u * 2048;
    o.p[4] = nullptr;
    o.p[5] = nullptr;
  }
  return o;
}

struct Item {
  int b, hg, split, tok0, tok1, page0, npages;
  int fill_to;  // splits split+1 .. fill_to-1 of the unit get empty partials from this item
};

// Valid tokens of this launch: the host's T, or the device-side length (a
// launch captured once and replayed while the cache grows), clamped to the
// capacity the plan was made for.
__device__ __forceinline__ int valid_tokens(const AttnArgs& a, int b) {
  if (a.T_dev == nullptr) return a.T;
  return max(0, min(a.T, a.T_dev[static_cast<int64_t>(b) * a.T_stride] + a.T_add));
}

// An item whose split lies past its sequence's length has no pages: its warps
// write an empty partial (m = -inf, l = 0, o = 0), which the merge weighs with 0.
// With device lengths the plan fixes only the number of splits: sequence b's
// splits are runs of ceil(ceil(T_b / 16) / ns) pages, so the work stays
// balanced however far the cache is from the capacity the plan was made for.
// The cache page holding page pg of sequence b; -1 when a block-table entry is
// outside the pool (nothing of it is read: its TMA boxes start at a negative
// row and fill with zeros, and the metadata is skipped; the status word gets
// EXK_S_PAGE_INDEX).
__device__ __forceinline__ int page_of(const AttnArgs& a, int b, int pg) {
  if (a.pages == nullptr) return b * a.NP + pg;
  const int p = __ldg(a.pages + static_cast<int64_t>(b) * a.pages_stride + pg);
  if (p < 0 || p >= a.pool_pages) {
    set_status(a.status, EXK_S_PAGE_INDEX);
    return -1;
  }
  return p;
}

__device__ __forceinline__ int item_split_len(const AttnArgs& a, int T) {
  if (a.T_dev == nullptr) return a.split_len;
  return max(1, ((T + kP - 1) / kP + a.ns - 1) / a.ns) * kP;
}

template <int WPH>
__device__ __forceinline__ Item decode_item(const AttnArgs& a, int item) {
  Item it;
  if (a.bal_G > 0) {
    const int64_t G = a.bal_G;
    int64_t W = a.bal_W, Su = a.bal_Su;
    int T = a.T;
    if (a.T_dev != nullptr) {
      // one device-side length for the batch: the partition follows it (a
      // length of 0 keeps one empty stage per unit, so every split is closed)
      T = valid_tokens(a, 0);
      Su = max(1, ((T + kP - 1) / kP + WPH - 1) / WPH);
      W = static_cast<int64_t>(a.B) * a.ngroups * Su;
    }
    // Quotients of products below 2^41 (W < 2^31 stages, G <= 1024 CTAs) in
    // double precision: the products are exact and the division is correctly
    // rounded; a non-integer c W / G lies at least 1/G from an integer and is
    // rounded by less than 2^-22, a non-integer (x + 1) G / W at least 1/W and
    // by less than 2^-42, so floor and ceil come out exact. (64-bit integer
    // divisions here cost ~1 us at every item start.)
    const int c = item % a.bal_G, j = item / a.bal_G;
    const double dW = static_cast<double>(W), dG = static_cast<double>(G);
    const int64_t lo = static_cast<int64_t>(static_cast<double>(c) * dW / dG);
    const int64_t hi = static_cast<int64_t>(static_cast<double>(c + 1) * dW / dG);
    const int64_t u = static_cast<int>(lo) / static_cast<int>(Su) + j;
    const int64_t s0 = max(lo, u * Su), s1 = min(hi, (u + 1) * Su);
    it.b = static_cast<int>(u) / a.ngroups;
    it.hg = static_cast<int>(u) % a.ngroups;
    if (s0 >= s1 || u * Su >= W) {  // past this CTA's run: no pages, no partial
      it.b = it.hg = 0;              // (u may lie past the last unit)
      it.split = -1;
      it.fill_to = -1;
      it.tok0 = it.tok1 = it.page0 = it.npages = 0;
      return it;
    }
    // the CTA whose run holds stage x (runs are empty where there are fewer stages than CTAs)
    auto owner = [&](int64_t x) { return static_cast<int64_t>(ceil(static_cast<double>(x + 1) * dG / dW)) - 1; };
    const int64_t first = owner(u * Su);
    it.split = static_cast<int>(c - first);
    // the piece closes the columns of the empty runs up to the unit's next
    // piece, and the unit's last piece every column after it
    it.fill_to = s1 == (u + 1) * Su ? a.ns : static_cast<int>(owner(s1) - first);
    it.tok0 = static_cast<int>((s0 - u * Su) * WPH * kP);
    it.tok1 = max(it.tok0, min(static_cast<int>((s1 - u * Su) * WPH * kP), T));
    it.page0 = it.tok0 / kP;
    it.npages = (it.tok1 - it.tok0 + kP - 1) / kP;
    return it;
  }
  const int bg = item / a.nsl;
  it.split = a.s0 + item % a.nsl;
  it.fill_to = it.split + 1;
  it.b = bg / a.ngroups;
  it.hg = bg % a.ngroups;
  const int T = valid_tokens(a, it.b);
  const int sl = item_split_len(a, T);
  it.tok0 = it.split * sl;
  it.tok1 = max(it.tok0, min(it.tok0 + sl, T));
  it.page0 = it.tok0 / kP;
  it.npages = (it.tok1 - it.tok0 + kP - 1) / kP;
  return it;
}

// ------------------------------------------------------------------ fragment loaders
//
// Lane (g = lane/4, t = lane%4).
// K (A operand of S^T = K Q^T): rows sigma(g), sigma(g)+8; mma kk (0..7)
//   covers channel quad 16t+4kk (kk<4) or 64+16t+4(kk-4); kw[row][2kk] holds
//   the quad's channels 0-1, kw[row][2kk+1] channels 2-3 (bf16 pairs).
// V (A operand of O^T = V^T P^T): token pairs (sigma(2t), sigma(2t+1)) and
//   the same +8; m-tile mm covers channels chA = v_channel(mm, g) and chB =
//   chA+1 (bf16 kernel: 8g+2mm (mm<4) or 64+8g+2(mm-4); compressed kernel:
//   16mm+2g, see load_v_comp); vw[pair][mm][0] = (V[tokA][chA], V[tokB][chA]),
//   vw[pair][mm][1] the same for chB.

// KKILL = false: the page's K base bytes have no zero group (checked by the
// caller), so the code-0 rule is skipped.
template <bool KKILL = true>
__device__ __forceinline__ void load_k_comp(const Slot& s, int g, int t, uint32_t (&kw)[2][16]) {
  const uint8_t* sm = s.p[0];
  const uint8_t* cd = s.p[1];
  const uint8_t* bs = s.p[2];
  const uint4 bl = *reinterpret_cast<const uint4*>(bs + 16 * t);
  const uint4 bh = *reinterpret_cast<const uint4*>(bs + 64 + 16 * t);
  const uint32_t bw[8] = {bl.x, bl.y, bl.z, bl.w, bh.x, bh.y, bh.z, bh.w};
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = sigma(g) + 8 * rr;
    const int sw = r & 7, cs = (r >> 1) & 3;
    const uint4 sl = *reinterpret_cast<const uint4*>(sm + r * 128 + ((t ^ sw) << 4));
    const uint4 sh = *reinterpret_cast<const uint4*>(sm + r * 128 + (((t + 4) ^ sw) << 4));
    const uint4 cw = *reinterpret_cast<const uint4*>(cd + r * 64 + ((t ^ cs) << 4));
    const uint32_t smw[8] = {sl.x, sl.y, sl.z, sl.w, sh.x, sh.y, sh.z, sh.w};
    const uint32_t cwv[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t adj_lo = KKILL ? bw[kk] & 0x7F7F7F7Fu : bw[kk];
      const uint32_t adj_hi = KKILL ? bw[kk + 4] & 0x7F7F7F7Fu : bw[kk + 4];
      dec4f<KKILL, false, 0x5140u, 0x7362u>(smw[kk], cwv[kk], adj_lo, bw[kk], kw[rr][2 * kk], kw[rr][2 * kk + 1]);
      dec4f<KKILL, true, 0x5140u, 0x7362u>(smw[kk + 4], cwv[kk], adj_hi, bw[kk + 4], kw[rr][2 * kk + 8],
                                           kw[rr][2 * kk + 9]);
    }
  }
}

__device__ __forceinline__ void load_k_bf16(const Slot& s, int g, int t, uint32_t (&kw)[2][16]) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = sigma(g) + 8 * rr;
    const int sw = r & 7;
    const uint8_t* lo = s.p[0] + r * 128;
    const uint8_t* hi = s.p[1] + r * 128;
    const uint4 a = *reinterpret_cast<const uint4*>(lo + (((2 * t) ^ sw) << 4));
    const uint4 b = *reinterpret_cast<const uint4*>(lo + (((2 * t + 1) ^ sw) << 4));
    const uint4 c = *reinterpret_cast<const uint4*>(hi + (((2 * t) ^ sw) << 4));
    const uint4 d = *reinterpret_cast<const uint4*>(hi + (((2 * t + 1) ^ sw) << 4));
    const uint32_t w[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) kw[rr][i] = w[i];
  }
}

// Compressed V through ldmatrix.trans. The bytes of the sm and code tiles are
// read as b16 elements (two channels each), so a transposed 8x8 load gives lane
// (g, t) the word [A(ch), A(ch+1), B(ch), B(ch+1)] of tokens A, B (the matrix
// rows 2t, 2t+1) and channels ch = 16c + 2g, ch + 1 of 16-byte chunk c — the
// token pair of a V^T fragment with no byte interleaving, and the base bytes
// come duplicated per token ([b(ch), b(ch+1), b(ch), b(ch+1)]) from a matrix
// whose eight row addresses are all the chunk of the base row. m-tile c of
// O^T = V^T P^T then holds channel 16c + 2g in row g and 16c + 2g + 1 in row
// g + 8 (v_channel). Matrix row j of token half pp is page token sigma(j) + 8pp,
// the token order of P^T.
struct VOffs {
  uint32_t sm[4];  // sm tile:   load k -> chunks 2k, 2k+1 (x token halves 0, 1)
  uint32_t cd[2];  // code tile: load k -> chunks 2k, 2k+1 (x token halves)
  uint32_t bs[2];  // base row:  load k -> chunks 4k .. 4k+3
};

__device__ __forceinline__ VOffs v_offsets(int lane) {
  const int mi = lane >> 3, ri = lane & 7;
  const int row = sigma(ri) + 8 * (mi & 1);
  VOffs o;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = 2 * k + (mi >> 1);
    o.sm[k] = static_cast<uint32_t>(row * 128 + ((c ^ (row & 7)) << 4));
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int c = 2 * k + (mi >> 1);
    o.cd[k] = static_cast<uint32_t>(row * 64 + ((c ^ ((row >> 1) & 3)) << 4));
    o.bs[k] = static_cast<uint32_t>(16 * (4 * k + mi));
  }
  return o;
}

// Channel of row g of V m-tile c (row g + 8 holds the next channel).
template <bool COMP>
__device__ __forceinline__ int v_channel(int c, int g) {
  if constexpr (COMP) return 16 * c + 2 * g;
  return c < 4 ? 8 * g + 2 * c : 64 + 8 * g + 2 * (c - 4);
}

// The V base words of a page: eb[c] = [b(16c+2g), b(16c+2g+1)] twice.
__device__ __forceinline__ void load_v_base(const Slot& s, const VOffs& vo, uint32_t (&eb)[8]) {
  const uint32_t bs = smem_addr(s.p[5]);
  ldsm_x4_t(bs + vo.bs[0], eb[0], eb[1], eb[2], eb[3]);
  ldsm_x4_t(bs + vo.bs[1], eb[4], eb[5], eb[6], eb[7]);
}

// VKILL = false: the page's V base bytes have no zero group (checked by the
// caller), so the code-0 rule is skipped and the base bytes are used as they are.
template <bool VKILL>
__device__ __forceinline__ void load_v_comp(const Slot& s, const VOffs& vo, const uint32_t (&eb)[8],
                                            uint32_t (&vw)[2][8][2]) {
  const uint32_t sm = smem_addr(s.p[3]), cd = smem_addr(s.p[4]);
  uint32_t smr[2][8], cdr[2][4];  // [token half][chunk]
#pragma unroll
  for (int k = 0; k < 4; ++k) ldsm_x4_t(sm + vo.sm[k], smr[0][2 * k], smr[1][2 * k], smr[0][2 * k + 1], smr[1][2 * k + 1]);
#pragma unroll
  for (int k = 0; k < 2; ++k) ldsm_x4_t(cd + vo.cd[k], cdr[0][2 * k], cdr[1][2 * k], cdr[0][2 * k + 1], cdr[1][2 * k + 1]);
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      dec4f<VKILL, false, 0x6240u, 0x7351u>(smr[pp][c], cdr[pp][c], VKILL ? eb[c] & 0x7F7F7F7Fu : eb[c], eb[c],
                                            vw[pp][c][0], vw[pp][c][1]);
      dec4f<VKILL, true, 0x6240u, 0x7351u>(smr[pp][c + 4], cdr[pp][c], VKILL ? eb[c + 4] & 0x7F7F7F7Fu : eb[c + 4],
                                           eb[c + 4], vw[pp][c + 4][0], vw[pp][c + 4][1]);
    }
  }
}

__device__ __forceinline__ void load_v_bf16(const Slot& s, int g, int t, uint32_t (&vw)[2][8][2]) {
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const int ra = sigma(2 * t) + 8 * pp;
    const int rb = sigma(2 * t + 1) + 8 * pp;
    const uint4 al = *reinterpret_cast<const uint4*>(s.p[2] + ra * 128 + ((g ^ (ra & 7)) << 4));
    const uint4 ah = *reinterpret_cast<const uint4*>(s.p[3] + ra * 128 + ((g ^ (ra & 7)) << 4));
    const uint4 bl = *reinterpret_cast<const uint4*>(s.p[2] + rb * 128 + ((g ^ (rb & 7)) << 4));
    const uint4 bh = *reinterpret_cast<const uint4*>(s.p[3] + rb * 128 + ((g ^ (rb & 7)) << 4));
    const uint32_t aw[8] = {al.x, al.y, al.z, al.w, ah.x, ah.y, ah.z, ah.w};
    const uint32_t bw[8] = {bl.x, bl.y, bl.z, bl.w, bh.x, bh.y, bh.z, bh.w};
#pragma unroll
    for (int mm = 0; mm < 8; ++mm) {
      vw[pp][mm][0] = prmt(aw[mm], bw[mm], 0x5410u);
      vw[pp][mm][1] = prmt(aw[mm], bw[mm], 0x7632u);
    }
  }
}

// The raw rows of one page-tile: row j (its rank among the page's raw rows)
// at p + j * 128, for j < lim. p is the stage's shared-memory copy made by
// the producer, or the global pool when the rows were not staged.
struct RawRows {
  const uint16_t* p;
  int lim;
};

// Row of raw token `r` of a page, or nullptr (and a status) when the
// metadata points outside the pool.
__device__ __forceinline__ const uint4* raw_row(uint32_t rm, const RawRows& src, int r, int32_t* status) {
  const int j = __popc(rm & ((1u << r) - 1u));
  if (src.p == nullptr || j >= src.lim) {
    set_status(status, EXK_S_RAW_INDEX);
    return nullptr;
  }
  return reinterpret_cast<const uint4*>(src.p + static_cast<int64_t>(j) * kD);
}

// Rows flagged in `fl` are replaced: raw rows (bit set in rm) by their pool
// row, rows past the valid tokens by zeros (the reference loads them as 0).
__device__ __forceinline__ void fix_k_rows(uint32_t fl, uint32_t rm, const RawRows& src, int32_t* status, int vr,
                                           int g, int t, uint32_t (&kw)[2][16]) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = sigma(g) + 8 * rr;
    if ((fl >> r) & 1u) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = 0u;
      if (r < vr && ((rm >> r) & 1u)) {
        const uint4* row = raw_row(rm, src, r, status);
        if (row != nullptr) {
          const uint4 a = row[2 * t], b = row[2 * t + 1], c = row[8 + 2 * t], d = row[8 + 2 * t + 1];
          const uint32_t x[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = x[i];
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) kw[rr][i] = w[i];
    }
  }
}

__device__ __forceinline__ void raw_v_words(uint32_t fl, uint32_t rm, const RawRows& src, int32_t* status, int vr,
                                            int r, int g, uint32_t (&w)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = 0u;
  if (((fl >> r) & 1u) && r < vr && ((rm >> r) & 1u)) {
    const uint4* row = raw_row(rm, src, r, status);
    if (row != nullptr) {
      const uint4 a = row[g], b = row[8 + g];
      w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
  }
}

__device__ __forceinline__ void fix_v_rows(uint32_t fl, uint32_t rm, const RawRows& src, int32_t* status, int vr,
                                           int g, int t, uint32_t (&vw)[2][8][2]) {
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const int ra = sigma(2 * t) + 8 * pp;
    const int rb = sigma(2 * t + 1) + 8 * pp;
    const bool fa = (fl >> ra) & 1u, fb = (fl >> rb) & 1u;
    if (fa || fb) {
      uint32_t wa[8], wb[8];
      raw_v_words(fl, rm, src, status, vr, ra, g, wa);
      raw_v_words(fl, rm, src, status, vr, rb, g, wb);
      const uint32_t mask = (fa ? 0x0000FFFFu : 0u) | (fb ? 0xFFFF0000u : 0u);
#pragma unroll
      for (int mm = 0; mm < 8; ++mm) {
        const uint32_t n0 = prmt(wa[mm], wb[mm], 0x5410u);
        const uint32_t n1 = prmt(wa[mm], wb[mm], 0x7632u);
        vw[pp][mm][0] = (vw[pp][mm][0] & ~mask) | (n0 & mask);
        vw[pp][mm][1] = (vw[pp][mm][1] & ~mask) | (n1 & mask);
      }
    }
  }
}

// Row r of V (its 256-byte bf16 row at `row`, or zeros when row is null)
// written into the ldmatrix-layout fragments of the compressed kernel: the
// lane's word for chunk c is the channel pair (16c + 2g, 16c + 2g + 1); token
// A of the pair takes the low halves, token B the high halves.
__device__ __forceinline__ void put_v_row_t(const uint32_t* row, bool b_side, int g, uint32_t (&v)[8][2]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t w = row != nullptr ? row[8 * c + g] : 0u;
    if (b_side) {
      v[c][0] = prmt(w, v[c][0], 0x1054u);
      v[c][1] = prmt(w, v[c][1], 0x3254u);
    } else {
      v[c][0] = prmt(w, v[c][0], 0x7610u);
      v[c][1] = prmt(w, v[c][1], 0x7632u);
    }
  }
}

// The compressed kernel's V fix-up (ldmatrix layout): rows flagged in `fl`
// are replaced, raw rows (bit set in rm) by their pool row, rows past the
// valid tokens by zeros.
__device__ __forceinline__ void fix_v_rows_t(uint32_t fl, uint32_t rm, const RawRows& src, int32_t* status, int vr,
                                             int g, int t, uint32_t (&vw)[2][8][2]) {
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
#pragma unroll
    for (int ab = 0; ab < 2; ++ab) {
      const int r = sigma(2 * t + ab) + 8 * pp;
      if ((fl >> r) & 1u) {
        const uint4* row = (r < vr && ((rm >> r) & 1u)) ? raw_row(rm, src, r, status) : nullptr;
        put_v_row_t(reinterpret_cast<const uint32_t*>(row), ab != 0, g, vw[pp]);
      }
    }
  }
}

// ------------------------------------------------------------------ per-warp state

template <int NT>
struct WarpState {
  float m[NT][2];   // running max of the lane's two heads (2t, 2t+1) per n-tile
  float l[NT][2];   // lane-partial sum of exp2(s - m) over the lane's rows
  float acc[NT][8][4];
};

struct PageMeta {
  uint32_t rm[2];        // rowmask K, V
  uint32_t tag[2];       // staged position of the page's first raw row of K, V (0xFF: not staged)
  const uint16_t* area;  // the stage's raw area
  RawRows src[2];        // general body: where the page's raw rows of K, V are read
};

// Staged raw rows of a full page (see the producer): the lanes whose fragment
// rows are raw replace them with shared-memory loads. rm: rowmask; area: the
// stage's raw area (kRawRows rows); tag: the page's first staged row in it.
// Positions wrap inside the area, so no address can leave it.
template <int R>
__device__ __forceinline__ const uint4* staged_row(const uint16_t* area, uint32_t tag, uint32_t rm, int r) {
  static_assert((R & (R - 1)) == 0, "the raw area holds a power of two of rows");
  return reinterpret_cast<const uint4*>(area + ((tag + __popc(rm & ((1u << r) - 1u))) & (R - 1)) * kD);
}

template <int R>
__device__ __forceinline__ void patch_k_staged(uint32_t rm, uint32_t tag, const uint16_t* area, int g, int t,
                                               uint32_t (&kw)[2][16]) {
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = sigma(g) + 8 * rr;
    if ((rm >> r) & 1u) {
      const uint4* row = staged_row<R>(area, tag, rm, r);
      const uint4 a = row[2 * t], b = row[2 * t + 1], c = row[8 + 2 * t], d = row[8 + 2 * t + 1];
      const uint32_t x[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) kw[rr][i] = x[i];
    }
  }
}

template <int R>
__device__ __forceinline__ void patch_v_staged_t(uint32_t rm, uint32_t tag, const uint16_t* area, int g, int t,
                                                 uint32_t (&vw)[2][8][2]) {
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
#pragma unroll
    for (int ab = 0; ab < 2; ++ab) {
      const int r = sigma(2 * t + ab) + 8 * pp;
      if ((rm >> r) & 1u)
        put_v_row_t(reinterpret_cast<const uint32_t*>(staged_row<R>(area, tag, rm, r)), ab != 0, g, vw[pp]);
    }
  }
}

// Page bodies of the warp. kFast: a full page without raw rows (no fixup code
// at all, so nothing splits the decode / mma schedule). kStaged: a full page
// whose raw rows were all staged in shared memory by the producer; the lanes
// whose rows are raw patch them in with shared-memory loads. Both need a V
// page without zero groups (V decodes without the code-0 rule). kGeneral:
// everything else — raw rows read from wherever the metadata says, rows past
// the valid tokens masked (a sequence's last partial page, staging out of
// room, zero groups in V).
enum PageMode { kFast = 0, kStaged = 1, kGeneral = 2 };

// Rescale the running output only when some row's maximum grew: with
// alpha = 1 exactly (ex2(0) = 1) the skipped multiplies would leave every bit as
// it is, so the result is the same either way. EXK_LAZY_RESCALE = 0 restores the
// unconditional rescale.
#ifndef EXK_LAZY_RESCALE
#define EXK_LAZY_RESCALE 1
#endif


// KKILL = false would skip K's code-0 rule on pages without a K zero group;
// every body keeps it (a second fast body for such pages measured 121 vs 90 us
// at 32x4096: the larger loop schedules worse).
template <bool COMP, int NT, int MODE, bool KKILL>
__device__ __forceinline__ void attend_page(const Slot& s, const PageMeta& pm, int vr, const AttnArgs& a,
                                            const uint32_t (&qf)[NT][16], WarpState<NT>& st, int g, int t,
                                            const VOffs& vo, const uint32_t (&eb)[8]) {
  const uint32_t tailmask = vr < kP ? (0xFFFFu & ~((1u << vr) - 1u)) : 0u;

  // ---- S^T = K . Q^T
  uint32_t kw[2][16];
  if constexpr (COMP) load_k_comp<KKILL>(s, g, t, kw); else load_k_bf16(s, g, t, kw);
  if constexpr (MODE == kGeneral) {
    const uint32_t fl = (COMP ? pm.rm[0] : 0u) | tailmask;
    if (fl != 0u) fix_k_rows(fl, pm.rm[0], pm.src[0], a.status, vr, g, t, kw);
  } else if constexpr (MODE == kStaged && COMP) {
    patch_k_staged<kRawArea>(pm.rm[0], pm.tag[0], pm.area, g, t, kw);
  }
  // two independent accumulation chains (low and high channel halves), summed
  float sc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float s1[4] = {0.f, 0.f, 0.f, 0.f};
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      mma_bf16(sc[nt], kw[0][2 * kk], kw[1][2 * kk], kw[0][2 * kk + 1], kw[1][2 * kk + 1], qf[nt][2 * kk],
               qf[nt][2 * kk + 1]);
      mma_bf16(s1, kw[0][2 * kk + 8], kw[1][2 * kk + 8], kw[0][2 * kk + 9], kw[1][2 * kk + 9], qf[nt][2 * kk + 8],
               qf[nt][2 * kk + 9]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[nt][i] += s1[i];
  }

  // ---- V fragments (issued before the softmax so the shared loads overlap it)
  uint32_t vw[2][8][2];
  if constexpr (COMP) {
    load_v_comp<MODE == kGeneral>(s, vo, eb, vw);
    if constexpr (MODE == kGeneral) {
      const uint32_t fl = pm.rm[1] | tailmask;
      if (fl != 0u) fix_v_rows_t(fl, pm.rm[1], pm.src[1], a.status, vr, g, t, vw);
    } else if constexpr (MODE == kStaged) {
      patch_v_staged_t<kRawArea>(pm.rm[1], pm.tag[1], pm.area, g, t, vw);
    }
  } else {
    load_v_bf16(s, g, t, vw);
    if constexpr (MODE == kGeneral) {
      if (tailmask != 0u) fix_v_rows(tailmask, 0u, pm.src[1], a.status, vr, g, t, vw);
    }
  }

  // ---- online softmax (base 2) over the page's 16 rows
  const int r0 = sigma(g), r1 = r0 + 8;
  uint32_t pb[NT][2];
  float alpha[NT][2];
  float p[NT][4];
  bool grew = false;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[nt][i] = sc[nt][i] * a.qk_scale;
    if constexpr (MODE == kGeneral) {
      if (r0 >= vr) p[nt][0] = p[nt][1] = -INFINITY;
      if (r1 >= vr) p[nt][2] = p[nt][3] = -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = fmaxf(p[nt][j], p[nt][2 + j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
      const float mn = fmaxf(st.m[nt][j], mx);
      grew |= mn != st.m[nt][j];
      alpha[nt][j] = mn;  // the new maximum until the rescale decision
    }
  }
  const bool rescale = EXK_LAZY_RESCALE ? __any_sync(0xFFFFFFFFu, grew) : true;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float mn = alpha[nt][j];
      alpha[nt][j] = rescale ? ex2(st.m[nt][j] - mn) : 1.0f;
      p[nt][j] = ex2(p[nt][j] - mn);
      p[nt][2 + j] = ex2(p[nt][2 + j] - mn);
      st.l[nt][j] = st.l[nt][j] * alpha[nt][j] + p[nt][j] + p[nt][2 + j];
      st.m[nt][j] = mn;
    }
    // P (rows = tokens, cols = heads) -> P^T fragments via 8x8 transposes
    pb[nt][0] = movmatrix_t(pack_bf16x2(p[nt][0], p[nt][1]));
    pb[nt][1] = movmatrix_t(pack_bf16x2(p[nt][2], p[nt][3]));
  }

  // ---- O^T = O^T * alpha + V^T . P^T
  if (rescale) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int mm = 0; mm < 8; ++mm) {
        float* c = st.acc[nt][mm];
        c[0] *= alpha[nt][0];
        c[1] *= alpha[nt][1];
        c[2] *= alpha[nt][0];
        c[3] *= alpha[nt][1];
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int mm = 0; mm < 8; ++mm)
      mma_bf16(st.acc[nt][mm], vw[0][mm][0], vw[0][mm][1], vw[1][mm][0], vw[1][mm][1], pb[nt][0], pb[nt][1]);
  }
}


template <int NT>
__device__ __forceinline__ void load_q(const AttnArgs& a, int b, int hk, int g, int t, uint32_t (&qf)[NT][16]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = nt * 8 + g;
    if (h < a.G) {
      const uint4* qr = reinterpret_cast<const uint4*>(a.q + (static_cast<int64_t>(b) * a.Hq + hk * a.G + h) * kD);
      const uint4 x0 = qr[2 * t], x1 = qr[2 * t + 1], x2 = qr[8 + 2 * t], x3 = qr[8 + 2 * t + 1];
      const uint32_t w[16] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w,
                              x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
#pragma unroll
      for (int i = 0; i < 16; ++i) qf[nt][i] = w[i];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) qf[nt][i] = 0u;
    }
  }
}

// ------------------------------------------------------------------ split merge

// Partials of one workspace: o [rows, ns, 128], m, l [rows, ns]; split s of
// the locator is column s0 + s.
struct WsSplits {
  const float* o_;
  const float* m_;
  const float* l_;
  int64_t row, ns, s0;
  __device__ const float* m(int s) const { return m_ + row * ns + s0 + s; }
  __device__ const float* l(int s) const { return l_ + row * ns + s0 + s; }
  __device__ const float4* o(int s) const { return reinterpret_cast<const float4*>(o_ + (row * ns + s0 + s) * kD); }
};

// Where a merged row goes. Bf16Out: the attention output, acc / den in bf16.
// PartialOut: the partial of the union of the merged splits, in the layout of
// one split's partial (o = acc unnormalised, m = the splits' maximum M, l =
// den), which a later merge combines with others like any split.
struct Bf16Out {
  uint16_t* row;
  __device__ void put(int lane, float4 acc, float den, float) const {
    uint2 r;
    r.x = pack_bf16x2(acc.x / den, acc.y / den);
    r.y = pack_bf16x2(acc.z / den, acc.w / den);
    reinterpret_cast<uint2*>(row)[lane] = r;
  }
};

struct PartialOut {
  float* o;
  float* m;
  float* l;
  __device__ void put(int lane, float4 acc, float den, float M) const {
    reinterpret_cast<float4*>(o)[lane] = acc;
    if (lane == 0) {
      *m = M;
      *l = den;
    }
  }
};

constexpr int kMaxRanks = 16;

// Partials of the `world` GPUs of a KV-sequence split: rank r's block (at
// base[r]: rows * nmax * 130 floats, rounded up to a multiple of 4) holds
// o [rows, nmax, 128], then m, l [rows, nmax]; its first cnt[r] splits are
// splits pre[r] .. pre[r] + cnt[r] - 1 of the whole sequence. The blocks are
// either in this GPU's memory (all-gathered) or read in place from the peers
// over NVLink; then `flags` is set and the merge first waits for the peers'
// signals (peers_ready).
struct GatherArgs {
  const float* base[kMaxRanks];
  int rows, nmax, world, ns;
  int pre[kMaxRanks + 1];
  uint32_t* flags;                 // this GPU's flag words, one per rank (nullptr: no exchange)
  uint32_t* peer_flag[kMaxRanks];  // word `rank` of peer p's flags
  uint32_t epoch;                  // the call's number, the same on every rank
  int rank;
  int32_t* status;
};

struct GatheredSplits {
  const GatherArgs* g;
  int64_t row;
  __device__ const float* base(int s, int& j) const {
    int r = 0;
    while (r + 1 < g->world && s >= g->pre[r + 1]) ++r;
    j = s - g->pre[r];
    return g->base[r];
  }
  __device__ const float* m(int s) const {
    int j;
    const float* b = base(s, j);
    return b + static_cast<int64_t>(g->rows) * g->nmax * kD + row * g->nmax + j;
  }
  __device__ const float* l(int s) const {
    int j;
    const float* b = base(s, j);
    return b + static_cast<int64_t>(g->rows) * g->nmax * (kD + 1) + row * g->nmax + j;
  }
  __device__ const float4* o(int s) const {
    int j;
    const float* b = base(s, j);
    return reinterpret_cast<const float4*>(b + (row * g->nmax + j) * kD);
  }
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The exchange of a peer merge, run by every CTA before it reads any block:
// publish this rank's epoch to every peer (the partials were written by the
// split kernel that ran before this kernel on the stream), then wait until
// every peer has published it too. Every CTA publishes (the stores are
// idempotent), so no CTA's wait depends on another CTA of this grid being
// resident. The wait gives up after kWaitLimitNs with EXK_S_PEER_TIMEOUT.
// A block is overwritten only two calls later (the caller alternates two
// blocks), by which time every peer has finished reading it: a rank starts
// call e + 2 only after its merge of call e + 1, which waited for every
// peer's signal of call e + 1, sent after that peer's merge of call e.
__device__ __forceinline__ bool peers_ready(const GatherArgs& g) {
  __shared__ int s_ok;
  if (threadIdx.x < g.world && static_cast<int>(threadIdx.x) != g.rank) {
    __threadfence_system();
    st_release_sys(g.peer_flag[threadIdx.x], g.epoch);
  }
  if (threadIdx.x == 0) {
    int ok = g.status == nullptr || *reinterpret_cast<volatile int32_t*>(g.status) == 0;
    for (int p = 0; ok && p < g.world; ++p) {
      if (p == g.rank) continue;
      if (static_cast<int32_t>(ld_acquire_sys(g.flags + p) - g.epoch) >= 0) continue;
      const uint64_t t0 = globaltimer();
      while (static_cast<int32_t>(ld_acquire_sys(g.flags + p) - g.epoch) < 0) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          set_status(g.status, EXK_S_PEER_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// out[row] = sum_s w_s o_s / sum_s w_s l_s with w_s = 2^(m_s - max_s m_s), by
// one warp (the reference's _reduce_kernel, exactkv/kernels.py:33-43), for up
// to kWideSplits = 16 splits: every load at once (one round trip; lane s holds
// split s's m and l), then the sums in split order. `loc` gives the addresses
// of split s of the row (m, l and the lane's float4 of o), so partials laid out
// by one workspace or gathered from several GPUs merge with the same
// arithmetic, bit for bit.
template <class Loc, class Out>
__device__ __forceinline__ void merge_row(const Loc& loc, int ns, int lane, const Out& out) {
  const float mv = lane < ns ? __ldcg(loc.m(lane)) : -INFINITY;
  const float lv = lane < ns ? __ldcg(loc.l(lane)) : 0.f;
  float4 v[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) v[u] = u < ns ? __ldcg(loc.o(u) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
  float M = mv;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, d));
  // an empty split (m = -inf) weighs 0, also when every split is empty
  const float w = lane < ns && mv != -INFINITY ? ex2(mv - M) : 0.f;
  float den = lane < ns ? w * lv : 0.f;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, d);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const float wu = __shfl_sync(0xFFFFFFFFu, w, u);
    if (u < ns) {
      acc.x += wu * v[u].x;
      acc.y += wu * v[u].y;
      acc.z += wu * v[u].z;
      acc.w += wu * v[u].w;
    }
  }
  out.put(lane, acc, den, M);
}

// Splits above which a row is merged by a whole CTA instead of one warp.
constexpr int kWideSplits = 16;
constexpr int kWideMaxWarps = 32;
constexpr int kChunk = 8;  // splits one warp loads at once

// Warps of the CTA that merges one row of ns > kWideSplits splits: one chunk
// of kChunk splits each, 2 to 32 warps (more splits: each warp takes several).
__host__ __device__ constexpr int wide_warps(int ns) {
  return (ns + kChunk - 1) / kChunk < 2 ? 2
         : ((ns + kChunk - 1) / kChunk > kWideMaxWarps ? kWideMaxWarps : (ns + kChunk - 1) / kChunk);
}

// merge_row for many splits (ns > kWideSplits), by the nw = wide_warps(ns)
// warps of the CTA in one memory round trip per chunk: warp w loads chunks w,
// w + nw, ... of kChunk splits (m, l and the o rows together), folds each
// into its running (max, sum of weights x l, sum of weights x o) in chunk
// order, rescaling by 2^(old max - new max) when the max grows; warp 0 then
// combines the warps in warp order, each scaled by 2^(its max - the row's).
// Splits with m = -inf (past a sequence's length) weigh 0. The order depends
// only on ns, so every caller with the same splits gets the same bits.
template <class Loc, class Out>
__device__ __forceinline__ void merge_row_wide(const Loc& loc, int ns, const Out& out) {
  __shared__ float s_max[kWideMaxWarps], s_den[kWideMaxWarps];
  __shared__ float4 s_acc[kWideMaxWarps][32];
  const int nw = wide_warps(ns);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float mw = -INFINITY, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = warp * kChunk; c0 < ns; c0 += nw * kChunk) {
    const int n = min(kChunk, ns - c0);
    const float mv = lane < n ? __ldcg(loc.m(c0 + lane)) : -INFINITY;
    const float lv = lane < n ? __ldcg(loc.l(c0 + lane)) : 0.f;
    float4 v[kChunk];
#pragma unroll
    for (int u = 0; u < kChunk; ++u) v[u] = u < n ? __ldcg(loc.o(c0 + u) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    float cm = mv;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xFFFFFFFFu, cm, d));
    const float mn = fmaxf(mw, cm);
    const float sc = mw == mn ? 1.f : ex2(mw - mn);  // mw = -inf < mn: 0
    const float w = mv == -INFINITY ? 0.f : ex2(mv - mn);
    float lw = w * lv;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) lw += __shfl_xor_sync(0xFFFFFFFFu, lw, d);
    den = den * sc + lw;
    acc.x *= sc;
    acc.y *= sc;
    acc.z *= sc;
    acc.w *= sc;
#pragma unroll
    for (int u = 0; u < kChunk; ++u) {
      const float wu = __shfl_sync(0xFFFFFFFFu, w, u);
      acc.x += wu * v[u].x;
      acc.y += wu * v[u].y;
      acc.z += wu * v[u].z;
      acc.w += wu * v[u].w;
    }
    mw = mn;
  }
  s_acc[warp][lane] = acc;
  if (lane == 0) {
    s_max[warp] = mw;
    s_den[warp] = den;
  }
  __syncthreads();
  if (warp != 0) return;
  float M = -INFINITY;
  for (int i = 0; i < nw; ++i) M = fmaxf(M, s_max[i]);
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
  den = 0.f;
  for (int i = 0; i < nw; ++i) {
    const float mi = s_max[i];
    const float f = mi == -INFINITY ? 0.f : ex2(mi - M);
    const float4 t = s_acc[i][lane];
    acc.x += f * t.x;
    acc.y += f * t.y;
    acc.z += f * t.z;
    acc.w += f * t.w;
    den += f * s_den[i];
  }
  out.put(lane, acc, den, M);
}

// ------------------------------------------------------------------ kernel

template <bool COMP, int NT, int NWC, int HG>
__global__ void __launch_bounds__((NWC + 1) * 32, 1)
    attn_split_kernel(const __grid_constant__ AttnArgs a, const __grid_constant__ AttnMaps tm) {
  using C = Cfg<COMP, NT, NWC, HG>;
  constexpr int S = C::kStages;
  constexpr int WPH = C::kWph;
  constexpr int H8 = C::kHeads;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align by offsetting the __shared__ array itself (not through an integer
  // round trip), so every access below stays a shared-memory access (LDS/STS)
  // rather than a generic one.
  uint8_t* ring = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  // raw rows of every stage, copied by the producer: [slot][kRawRows][128] bf16
  uint16_t* rawbuf = reinterpret_cast<uint16_t*>(ring + C::kRingBytes);
  float* macc = reinterpret_cast<float*>(ring + C::kRingBytes + S * C::kRawSlot);
  float* mbuf = reinterpret_cast<float*>(ring + C::kRingBytes + S * C::kRawSlot + C::kMergeBytes);
  float* lbuf = mbuf + NWC * H8;
  // page metadata of every stage, written by the producer: [slot][tile] = (rowmask K, rowoff K, rowmask V, rowoff V)
  int4* meta = reinterpret_cast<int4*>(lbuf + NWC * H8);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(meta) + S * C::kMetaSlot);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    // a merge launched as a programmatic dependent may start its (waiting) CTAs now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NWC);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NWC) {
    // ------------------------------------------------ producer warp
    // Per stage: lane 0 issues the tiles' TMA copies; lane u < NWC holds tile
    // u's page metadata (rowmask K, rowoff K, rowmask V, rowoff V), loaded one
    // stage ahead; lanes 2u + kv stage tile u's raw rows of cache kv into the
    // stage's raw area (positions from a warp prefix sum; bulk copies that
    // complete on the stage's barrier) while it has room, and bits 16-23 of the
    // rowmask the consumers read give the staged position (0xFF: read the pool).
    // The metadata goes beside the stage; lane 0's arrive releases it.
    if (lane == 0) {
      constexpr int nmaps = COMP ? 6 : 2;
      for (int i = 0; i < nmaps; ++i) prefetch_tmap(&tm.m[i]);
    }
    // phys: lane 0's cache page of the stage's first page (its TMA row / 16)
    auto tile_meta = [&](const Item& it_, int s_, int& phys) {
      int4 r = make_int4(0, 0, 0, 0);
      const int page = it_.page0 + s_ * WPH + lane % WPH;
      const int cp = (lane < NWC && page < it_.page0 + it_.npages) ? page_of(a, it_.b, page) : -1;
      phys = a.pages == nullptr ? it_.b * a.NP + it_.page0 + s_ * WPH : __shfl_sync(0xFFFFFFFFu, cp, 0);
      if constexpr (COMP) {
        if (cp >= 0) {
          const int64_t idx = static_cast<int64_t>(cp) * a.Hkv + it_.hg * HG + lane / WPH;
          r = make_int4(__ldg(a.rowmask[0] + idx), __ldg(a.rowoff[0] + idx), __ldg(a.rowmask[1] + idx),
                        __ldg(a.rowoff[1] + idx));
        }
      }
      return r;
    };
    int item = blockIdx.x, s = 0, nst = 0;
    Item it{};
    // the cursor skips items without pages (splits past the valid length)
    for (; item < a.n_items; item += gridDim.x) {
      it = decode_item<WPH>(a, item);
      nst = (it.npages + WPH - 1) / WPH;
      if (nst > 0) break;
    }
    int mphys = 0;
    int4 md = item < a.n_items ? tile_meta(it, 0, mphys) : make_int4(0, 0, 0, 0);
    uint32_t gs = 0;  // stages issued
    while (item < a.n_items) {
      const int slot = gs % S;
      const uint32_t round = gs / S;
      if (round > 0) {
        const bool w = mbar_wait(&empty[slot], (round - 1) & 1u);
        if (!__all_sync(0xFFFFFFFFu, w)) {
          if (lane == 0) {
            set_status(a.status, EXK_S_EMPTY_TIMEOUT);
            *abort_flag = 1;
          }
          break;
        }
      }
      if (__any_sync(0xFFFFFFFFu, *abort_flag != 0)) break;
      const int row = mphys * kP;  // -1 (outside the pool): a box of zeros
      const int h0 = it.hg * HG;
      uint8_t* st = ring + slot * C::kStageBytes;
      if constexpr (COMP) {
        if (lane == 0) {
          mbar_expect_tx(&full[slot], C::kTxBytes);
          const int prow = mphys;
          tma_load_3d(st, &tm.m[0], 0, row, h0, &full[slot]);
          tma_load_3d(st + NWC * 2048, &tm.m[3], 0, row, h0, &full[slot]);
          tma_load_3d(st + NWC * 4096, &tm.m[1], 0, row, h0, &full[slot]);
          tma_load_3d(st + NWC * 5120, &tm.m[4], 0, row, h0, &full[slot]);
          tma_load_3d(st + NWC * 6144, &tm.m[2], 0, prow, h0, &full[slot]);
          tma_load_3d(st + NWC * 6272, &tm.m[5], 0, prow, h0, &full[slot]);
        }
        const int tu = lane >> 1, kv = lane & 1;
        const int x = __shfl_sync(0xFFFFFFFFu, md.x, tu), y = __shfl_sync(0xFFFFFFFFu, md.y, tu);
        const int z = __shfl_sync(0xFFFFFFFFu, md.z, tu), w = __shfl_sync(0xFFFFFFFFu, md.w, tu);
        const uint32_t rm = static_cast<uint32_t>(kv ? z : x) & 0xFFFFu;
        const int ro = kv ? w : y;
        const int cnt = lane < 2 * NWC ? __popc(rm) : 0;
        int incl = cnt;  // inclusive prefix sum over the lanes
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
          if (lane >= d) incl += o;
        }
        const int off = incl - cnt;
        uint32_t tag = 0xFFu;
        if (cnt > 0 && incl <= C::kRawRows && ro >= 0 && static_cast<int64_t>(ro) + cnt <= a.raw_rows[kv]) {
          const uint32_t bytes = static_cast<uint32_t>(cnt) * kD * 2;
          mbar_expect_tx(&full[slot], bytes);
          bulk_g2s(rawbuf + (slot * C::kRawRows + off) * kD, a.raw[kv] + static_cast<int64_t>(ro) * kD, bytes,
                   &full[slot]);
          tag = static_cast<uint32_t>(off);
        }
        const int enc = static_cast<int>(rm | (tag << 16));
        const int ek = __shfl_sync(0xFFFFFFFFu, enc, (2 * lane) & 31);
        const int ev = __shfl_sync(0xFFFFFFFFu, enc, (2 * lane + 1) & 31);
        if (lane < NWC) meta[slot * NWC + lane] = make_int4(ek, md.y, ev, md.w);
        __syncwarp();  // every lane's stores and transaction counts come before the arrive
        if (lane == 0) mbar_arrive(&full[slot]);
      } else {
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[slot], C::kTxBytes);
          tma_load_3d(st, &tm.m[0], 0, row, h0, &full[slot]);
          tma_load_3d(st + NWC * 2048, &tm.m[0], 64, row, h0, &full[slot]);
          tma_load_3d(st + 2 * NWC * 2048, &tm.m[1], 0, row, h0, &full[slot]);
          tma_load_3d(st + 3 * NWC * 2048, &tm.m[1], 64, row, h0, &full[slot]);
        }
      }
      ++gs;
      if (++s == nst) {
        s = 0;
        for (item += gridDim.x; item < a.n_items; item += gridDim.x) {
          it = decode_item<WPH>(a, item);
          nst = (it.npages + WPH - 1) / WPH;
          if (nst > 0) break;
        }
      }
      if (item < a.n_items) md = tile_meta(it, s, mphys);  // the next stage's, in flight during the wait
    }
    // Every copy this warp issued lands before the CTA may exit.
    if (lane == 0) {
      for (uint32_t i = gs > S ? gs - S : 0; i < gs; ++i) {
        if (!mbar_wait(&full[i % S], (i / S) & 1u)) {
          set_status(a.status, EXK_S_DRAIN_TIMEOUT);
          break;
        }
      }
    }
    return;
  }

  // -------------------------------------------------- consumers: warp = (head hl, page phase ph)
  const int g = lane >> 2, t = lane & 3;
  const int hl = warp / WPH, ph = warp % WPH;
  const VOffs vo = v_offsets(lane);
  uint32_t gs = 0;
  bool aborted = false;
  WarpState<NT> st;
  uint32_t qf[NT][16];

  for (int item = blockIdx.x; item < a.n_items; item += gridDim.x) {
    const Item it = decode_item<WPH>(a, item);
    if (it.split < 0) continue;  // a balanced plan's empty piece: no pages, no partial
    const int hk = it.hg * HG + hl;
    const int nst = (it.npages + WPH - 1) / WPH;
    load_q<NT>(a, it.b, hk, g, t, qf);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      st.m[nt][0] = st.m[nt][1] = -INFINITY;
      st.l[nt][0] = st.l[nt][1] = 0.f;
#pragma unroll
      for (int mm = 0; mm < 8; ++mm) st.acc[nt][mm][0] = st.acc[nt][mm][1] = st.acc[nt][mm][2] = st.acc[nt][mm][3] = 0.f;
    }
    for (int s = 0; s < nst; ++s, ++gs) {
      const int p = s * WPH + ph;  // page of the item this warp takes from the stage
      const int slot = gs % S;
      if (!aborted) {
        if (*abort_flag) {
          aborted = true;
        } else if (!mbar_wait(&full[slot], (gs / S) & 1u)) {
          set_status(a.status, EXK_S_FULL_TIMEOUT);
          *abort_flag = 1;
          aborted = true;
        }
      }
      if (!aborted) {
        if (p < it.npages) {
          PageMeta pm;
          int4 v = make_int4(0, 0, 0, 0);
          if constexpr (COMP) v = meta[slot * NWC + warp];  // tile index hl * WPH + ph == warp
          pm.rm[0] = static_cast<uint32_t>(v.x) & 0xFFFFu;
          pm.rm[1] = static_cast<uint32_t>(v.z) & 0xFFFFu;
          pm.tag[0] = (static_cast<uint32_t>(v.x) >> 16) & 0xFFu;
          pm.tag[1] = (static_cast<uint32_t>(v.z) >> 16) & 0xFFu;
          pm.area = rawbuf + slot * C::kRawRows * kD;
          const int vr = min(kP, it.tok1 - (it.page0 + p) * kP);
          const Slot tl = tile_ptrs<COMP, NWC, HG>(ring + slot * C::kStageBytes, hl, ph);
          // warp-uniform choice of the page body
          bool vzero = false;
          uint32_t eb[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
          if constexpr (COMP) {
            load_v_base(tl, vo, eb);
            vzero = __any_sync(0xFFFFFFFFu, ((eb[0] | eb[1] | eb[2] | eb[3] | eb[4] | eb[5] | eb[6] | eb[7]) &
                                             0x80808080u) != 0u);
          }
          if ((pm.rm[0] | pm.rm[1]) == 0u && vr == kP && !vzero) {
            attend_page<COMP, NT, kFast, true>(tl, pm, vr, a, qf, st, g, t, vo, eb);
          } else if (COMP && vr == kP && !vzero && (pm.rm[0] == 0u || pm.tag[0] != 0xFFu) &&
                     (pm.rm[1] == 0u || pm.tag[1] != 0xFFu)) {
            attend_page<COMP, NT, kStaged, true>(tl, pm, vr, a, qf, st, g, t, vo, eb);
          } else {
#pragma unroll
            for (int kv = 0; kv < 2; ++kv) {
              const int ro = kv ? v.w : v.y;
              pm.src[kv].p = nullptr;
              pm.src[kv].lim = 0;
              if (!COMP) continue;
              if (pm.tag[kv] != 0xFFu) {
                pm.src[kv].p = pm.area + static_cast<int>(pm.tag[kv]) * kD;
                pm.src[kv].lim = __popc(pm.rm[kv]);
              } else if (ro >= 0 && ro < a.raw_rows[kv]) {
                pm.src[kv].p = a.raw[kv] + static_cast<int64_t>(ro) * kD;
                pm.src[kv].lim = a.raw_rows[kv] - ro < kP ? static_cast<int>(a.raw_rows[kv] - ro) : kP;
              }
            }
            attend_page<COMP, NT, kGeneral, true>(tl, pm, vr, a, qf, st, g, t, vo, eb);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }

    // splits of the unit that no CTA holds (a balanced plan): empty partials
    // (m = -inf, l = 0, o = 0), which the merge weighs with 0
    if (it.fill_to > it.split + 1 && ph == 0) {
      const int64_t r0 = static_cast<int64_t>(it.b) * a.Hq + static_cast<int64_t>(hk) * a.G;
      for (int h = 0; h < a.G; ++h)
        for (int sp = it.split + 1; sp < it.fill_to; ++sp) {
          const int64_t col = (r0 + h) * a.ns + sp;
          reinterpret_cast<float4*>(a.ws_o + col * kD)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (lane == 0) {
            a.ws_m[col] = -INFINITY;
            a.ws_l[col] = 0.f;
          }
        }
    }

    // ---- finish the item: full l per head, then (if several page phases) merge them
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float l = st.l[nt][j];
        l += __shfl_xor_sync(0xFFFFFFFFu, l, 4);
        l += __shfl_xor_sync(0xFFFFFFFFu, l, 8);
        l += __shfl_xor_sync(0xFFFFFFFFu, l, 16);
        st.l[nt][j] = l;
      }
    const int64_t row0 = static_cast<int64_t>(it.b) * a.Hq + static_cast<int64_t>(hk) * a.G;
    if constexpr (WPH == 1) {
      // one warp per head: the warp's state is the split partial
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = nt * 8 + 2 * t + j;
          if (h < a.G) {
            const int64_t col = (row0 + h) * a.ns + it.split;
            if (g == 0) {
              a.ws_m[col] = st.m[nt][j];
              a.ws_l[col] = st.l[nt][j];
            }
#pragma unroll
            for (int mm = 0; mm < 8; ++mm) {
              const int chA = v_channel<COMP>(mm, g);
              *reinterpret_cast<float2*>(a.ws_o + col * kD + chA) = make_float2(st.acc[nt][mm][j], st.acc[nt][mm][2 + j]);
            }
          }
        }
    } else {
      // WPH warps per head, merged in fixed phase order through shared memory
      named_barrier(1, NWC * 32);  // the previous item's readers are done
      if (g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            mbuf[warp * H8 + nt * 8 + 2 * t + j] = st.m[nt][j];
            lbuf[warp * H8 + nt * 8 + 2 * t + j] = st.l[nt][j];
          }
      }
      named_barrier(1, NWC * 32);
      float scale[NT][2];
      float lsum[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = nt * 8 + 2 * t + j;
          float M = -INFINITY;
#pragma unroll
          for (int q2 = 0; q2 < WPH; ++q2) M = fmaxf(M, mbuf[(hl * WPH + q2) * H8 + h]);
          const float mw = st.m[nt][j];
          scale[nt][j] = mw == -INFINITY ? 0.f : ex2(mw - M);
          float L = 0.f;
#pragma unroll
          for (int q2 = 0; q2 < WPH; ++q2) {
            const float m2 = mbuf[(hl * WPH + q2) * H8 + h];
            L += (m2 == -INFINITY ? 0.f : ex2(m2 - M)) * lbuf[(hl * WPH + q2) * H8 + h];
          }
          lsum[nt][j] = L;
          if (ph == 0) st.m[nt][j] = M;
        }
      float* buf = macc + hl * H8 * kAccPitch;
#pragma unroll 1
      for (int q2 = 0; q2 < WPH; ++q2) {
        if (ph == q2) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int mm = 0; mm < 8; ++mm) {
              const int chA = v_channel<COMP>(mm, g);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                float* r = buf + (nt * 8 + 2 * t + j) * kAccPitch + chA;
                float2 v = make_float2(scale[nt][j] * st.acc[nt][mm][j], scale[nt][j] * st.acc[nt][mm][2 + j]);
                if (q2 > 0) {
                  const float2 o = *reinterpret_cast<const float2*>(r);
                  v.x += o.x;
                  v.y += o.y;
                }
                if (q2 == WPH - 1) {
                  const int h = nt * 8 + 2 * t + j;
                  if (h < a.G) *reinterpret_cast<float2*>(a.ws_o + ((row0 + h) * a.ns + it.split) * kD + chA) = v;
                } else {
                  *reinterpret_cast<float2*>(r) = v;
                }
              }
            }
        }
        if (q2 < WPH - 1) named_barrier(1, NWC * 32);
      }
      if (ph == 0 && g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int h = nt * 8 + 2 * t + j;
            if (h < a.G) {
              const int64_t col = (row0 + h) * a.ns + it.split;
              a.ws_m[col] = st.m[nt][j];
              a.ws_l[col] = lsum[nt][j];
            }
          }
      }
    }

  }
}

// ------------------------------------------------------------------ merge

// WIDE = false: four rows per 128-thread CTA, one warp each; WIDE = true
// (ns > kWideSplits): one row per CTA of wide_warps(ns) warps.
template <bool WIDE>
__global__ void __launch_bounds__(WIDE ? kWideMaxWarps * 32 : 128)
    merge_kernel(const float* __restrict__ o, const float* __restrict__ m, const float* __restrict__ l, int ns,
                 int rows, uint16_t* __restrict__ out, int32_t* advance, int n_adv) {
  // Launched as a programmatic dependent of the split kernel: the CTAs may be
  // resident early; this waits until the split grid has finished and its
  // partials are visible (a no-op after an ordinary launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // a device-length step ends here: the split kernel has read the length
  if (advance != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *advance += n_adv;
  if constexpr (WIDE) {
    const int row = blockIdx.x;
    merge_row_wide(WsSplits{o, m, l, row, ns, 0}, ns, Bf16Out{out + static_cast<int64_t>(row) * kD});
  } else {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= rows) return;
    merge_row(WsSplits{o, m, l, row, ns, 0}, ns, threadIdx.x & 31, Bf16Out{out + static_cast<int64_t>(row) * kD});
  }
}

// The merge of the partials of the GPUs of a KV-sequence split (all-gathered
// into this GPU's memory, or read from the peers), in global split order (rank
// order, then each rank's own order).
template <bool WIDE>
__global__ void __launch_bounds__(WIDE ? kWideMaxWarps * 32 : 128)
    merge_gathered_kernel(const __grid_constant__ GatherArgs g, uint16_t* __restrict__ out) {
  // a programmatic dependent of the kernel before it (the split kernel, whose
  // partials must be complete before this rank signals its peers)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (g.flags != nullptr && !peers_ready(g)) return;
  if constexpr (WIDE) {
    const int row = blockIdx.x;
    merge_row_wide(GatheredSplits{&g, row}, g.ns, Bf16Out{out + static_cast<int64_t>(row) * kD});
  } else {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= g.rows) return;
    merge_row(GatheredSplits{&g, row}, g.ns, threadIdx.x & 31, Bf16Out{out + static_cast<int64_t>(row) * kD});
  }
}

// Splits [s0, s0 + n) of a workspace merged into one partial per row
// (PartialOut): po [rows, 128], pm, pl [rows].
template <bool WIDE>
__global__ void __launch_bounds__(WIDE ? kWideMaxWarps * 32 : 128)
    merge_partial_kernel(const float* __restrict__ o, const float* __restrict__ m, const float* __restrict__ l,
                         int ns, int s0, int n, int rows, float* __restrict__ po, float* __restrict__ pm,
                         float* __restrict__ pl) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (WIDE) {
    const int row = blockIdx.x;
    merge_row_wide(WsSplits{o, m, l, row, ns, s0}, n, PartialOut{po + static_cast<int64_t>(row) * kD, pm + row, pl + row});
  } else {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= rows) return;
    merge_row(WsSplits{o, m, l, row, ns, s0}, n, threadIdx.x & 31,
              PartialOut{po + static_cast<int64_t>(row) * kD, pm + row, pl + row});
  }
}


// ------------------------------------------------------------------ host side

namespace {

template <bool COMP, int NT, int NWC, int HG>
int launch_split(const AttnArgs& a, const AttnMaps& maps, int grid, int device, cudaStream_t stream) {
  using C = Cfg<COMP, NT, NWC, HG>;
  static bool configured[64] = {};
  auto kern = attn_split_kernel<COMP, NT, NWC, HG>;
  if (!configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[device] = true;
  }
  kern<<<grid, (NWC + 1) * 32, C::kBytes, stream>>>(a, maps);
  return launch_status();
}

template <bool COMP, int NT, int NWC>
int by_group(const AttnArgs& a, const AttnMaps& maps, int hg, int grid, int device, cudaStream_t stream) {
  switch (hg) {
    case 1: return launch_split<COMP, NT, NWC, 1>(a, maps, grid, device, stream);
    case 2: return launch_split<COMP, NT, NWC, 2>(a, maps, grid, device, stream);
    case 4: return launch_split<COMP, NT, NWC, 4>(a, maps, grid, device, stream);
    default:
      if constexpr (NWC >= 8) return launch_split<COMP, NT, NWC, 8>(a, maps, grid, device, stream);
      return EXK_EARG;
  }
}

template <bool COMP>
int dispatch_split(const AttnArgs& a, const AttnMaps& maps, int hg, int grid, int nwc, int device,
                   cudaStream_t stream) {
  const bool two = a.G > 8;
  if (nwc == 4) return two ? by_group<COMP, 2, 4>(a, maps, hg, grid, device, stream)
                           : by_group<COMP, 1, 4>(a, maps, hg, grid, device, stream);
  return two ? by_group<COMP, 2, 8>(a, maps, hg, grid, device, stream)
             : by_group<COMP, 1, 8>(a, maps, hg, grid, device, stream);
}

// Heads per CTA actually used: the plan's head group, capped by the consumer warps.
int cta_heads(int hkv, int nwc) { return std::min(head_group(hkv), nwc); }

// KV heads per work item: the plan's (ws->heads) when it sets one, else the
// default for Hkv; at most the consumer warps. -1 when the plan's is invalid.
int item_heads(const exk_partials* ws, int hkv, int nwc) {
  const int h = ws->heads;
  if (h == 0) return cta_heads(hkv, nwc);
  if ((h != 1 && h != 2 && h != 4 && h != 8) || hkv % h != 0) return -1;
  return std::min(h, nwc);
}

// Validates the shapes shared by both split kernels and fills AttnArgs.
int common_args(AttnArgs& a, const uint16_t* q, int B, int TS, int Hkv, int Hq, int T, int s0, int s1,
                const exk_partials* ws, int nwc, float qk_scale, int32_t* status) {
  if (ws == nullptr || q == nullptr) return EXK_EARG;
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || T <= 0 || TS <= 0 || TS % kP != 0 || T > TS) return EXK_EARG;
  if (Hq % Hkv != 0) return EXK_EARG;
  if (Hq / Hkv > 16) return EXK_EHEADS;
  if (nwc != 4 && nwc != 8) return EXK_EARG;
  const bool bal = ws->split_len == 0;  // a balanced plan (exk_plan_balanced): the whole call only
  if (ws->ns <= 0 || ws->split_len < 0 || ws->split_len % kP != 0) return EXK_EARG;
  if (bal && (s0 != 0 || s1 != ws->ns)) return EXK_EARG;
  if (!bal && static_cast<int64_t>(ws->ns) * ws->split_len < T) return EXK_EARG;
  if (s0 < 0 || s1 > ws->ns || s0 >= s1) return EXK_EARG;
  if (!bal && static_cast<int64_t>(s0) * ws->split_len >= T) return EXK_EARG;
  if (!aligned16(q) || !aligned16(ws->o)) return EXK_EALIGN;
  if (static_cast<int64_t>(B) * TS * Hkv > (int64_t{1} << 31) - 1) return EXK_EARG;
  a.q = q;
  a.ws_o = ws->o;
  a.ws_m = ws->m;
  a.ws_l = ws->l;
  a.status = status;
  a.B = B;
  a.TS = TS;
  a.NP = TS / kP;
  a.Hkv = Hkv;
  a.Hq = Hq;
  a.G = Hq / Hkv;
  a.T = T;
  a.T_dev = nullptr;
  a.T_add = 0;
  a.T_stride = 0;
  a.ns = ws->ns;
  a.split_len = ws->split_len;
  a.s0 = s0;
  // splits entirely past T (possible when s1 > the plan's last split) hold no work
  const int last = bal ? s1 - 1 : (T - 1) / ws->split_len;
  a.nsl = std::min(s1, last + 1) - s0;
  a.bal_G = 0;
  a.bal_Su = 0;
  a.bal_W = 0;
  const int hg = item_heads(ws, Hkv, nwc);
  if (hg <= 0) return EXK_EARG;
  a.ngroups = Hkv / hg;
  const int64_t items = static_cast<int64_t>(B) * a.ngroups * a.nsl;
  if (items > (int64_t{1} << 30)) return EXK_EARG;
  a.n_items = static_cast<int>(items);
  a.qk_scale = qk_scale;
  a.pages = nullptr;
  a.pages_stride = 0;
  a.pool_pages = 0;
  for (int i = 0; i < 2; ++i) {
    a.rowmask[i] = nullptr;
    a.rowoff[i] = nullptr;
    a.raw[i] = nullptr;
    a.raw_rows[i] = 0;
  }
  return 0;
}

// Tensor map over a [B*TS rows, H heads, width] buffer, addressed as
// (channel byte/element, token row, head): dims ordered so that a box of
// (width, rows, heads) lands head-major in shared memory ([heads][rows][width]).
int head_major_map(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int width, int elem_bytes, int64_t rows,
                   int H, int box_w, int box_rows, int box_heads, CUtensorMapSwizzle sw) {
  const uint64_t row_stride = static_cast<uint64_t>(width) * elem_bytes * H;
  const uint64_t head_stride = static_cast<uint64_t>(width) * elem_bytes;
  return make_tmap_3d(m, dt, ptr, width, rows, H, row_stride, head_stride, box_w, box_rows, box_heads, sw);
}

}  // namespace

}  // namespace exk

using namespace exk;

namespace {

// Best split of T tokens for items of hg KV heads (8 consumer warps, so a
// stage holds 8 / hg pages of each head). Cost of a candidate = (items on the
// busiest CTA) x (stages per item + a fixed per-item overhead of ~2 stages: Q
// load, pipeline refill, epilogue); returns that cost.
int64_t plan_for_heads(int B, int Hkv, int T, int num_ctas, int64_t hg, int32_t* ns_out, int32_t* sl_out) {
  const int64_t wph = 8 / hg;
  const int64_t npt = (T + kP - 1) / kP;
  const int64_t units = static_cast<int64_t>(B) * (Hkv / hg);
  constexpr int64_t kItemOverhead = 2;
  const int64_t nmax = std::min<int64_t>(npt, std::max<int64_t>(1, 8 * static_cast<int64_t>(num_ctas)));
  int64_t best_cost = -1, best_spp = npt;
  int64_t prev_spp = -1;
  for (int64_t n = 1; n <= nmax; ++n) {
    int64_t spp = (npt + n - 1) / n;
    spp = (spp + wph - 1) / wph * wph;  // whole stages per split
    if (spp == prev_spp) continue;
    prev_spp = spp;
    const int64_t nsr = (npt + spp - 1) / spp;
    if (nsr > 4096) break;
    const int64_t items = units * nsr;
    const int64_t waves = (items + num_ctas - 1) / num_ctas;
    const int64_t cost = waves * (spp / wph + kItemOverhead);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_spp = spp;
    }
  }
  *sl_out = static_cast<int32_t>(best_spp * kP);
  *ns_out = static_cast<int32_t>((npt + best_spp - 1) / best_spp);
  return best_cost;
}

}  // namespace

extern "C" int exk_plan_splits(int B, int Hkv, int T, int num_ctas, int32_t* ns_out, int32_t* sl_out) {
  if (B <= 0 || Hkv <= 0 || T <= 0 || num_ctas <= 0 || ns_out == nullptr || sl_out == nullptr) return EXK_EARG;
  // Items are (sequence, head group of up to 8 heads, split).
  plan_for_heads(B, Hkv, T, num_ctas, head_group(Hkv), ns_out, sl_out);
  return 0;
}

namespace {

// The balanced partition of a launch: units of Su stages, cut into G equal runs
// (W = units * Su < 2^31 stages and G <= kMaxBalancedCtas, which keep the
// kernel's double-precision quotients exact).
constexpr int64_t kMaxBalancedCtas = 1024;
struct Balance {
  int64_t units, Su, W, G;
  int splits;    // most pieces one unit is cut into (the workspace columns needed)
  int pieces;    // most pieces one CTA's run holds (items per CTA)
};

Balance balance_of(int B, int ngroups, int T, int wph, int ctas) {
  Balance b;
  b.units = static_cast<int64_t>(B) * ngroups;
  const int64_t npt = (T + kP - 1) / kP;
  b.Su = (npt + wph - 1) / wph;
  b.W = b.units * b.Su;
  // every CTA, also with fewer stages than CTAs (runs of 0 or 1 stage), as in a
  // device-length call, which cuts a length the host does not know
  b.G = ctas;
  auto lo = [&](int64_t c) { return c * b.W / b.G; };
  auto owner = [&](int64_t x) { return ((x + 1) * b.G + b.W - 1) / b.W - 1; };  // the CTA whose run holds stage x
  b.splits = 1;
  for (int64_t u = 0; u < b.units; ++u)
    b.splits = static_cast<int>(std::max<int64_t>(b.splits, owner((u + 1) * b.Su - 1) - owner(u * b.Su) + 1));
  b.pieces = 1;
  for (int64_t c = 0; c < b.G; ++c)
    b.pieces = static_cast<int>(std::max<int64_t>(b.pieces, (lo(c + 1) - 1) / b.Su - lo(c) / b.Su + 1));
  return b;
}

// Fills the balanced partition of a whole-call launch (ws->split_len == 0):
// contiguous caches, a host-side length or one device-side length for the
// batch; the grid is then exactly bal_G.
int balance_args(AttnArgs& a, const exk_partials* ws, int hg, int wph, int sms) {
  if (ws->split_len != 0) return 0;
  if (a.pages != nullptr || (a.T_dev != nullptr && a.T_stride != 0)) return EXK_EARG;
  if (a.T_dev != nullptr) {
    // the length is read on the device: bounds that hold for every length up
    // to the capacity a.T (a unit of Su stages spans at most ceil(G / units) + 1
    // runs, a run of W / G stages touches at most ceil(units / G) + 1 units)
    const int64_t units = static_cast<int64_t>(a.B) * (a.Hkv / hg);
    const int64_t G = sms;
    const int64_t splits = (G + units - 1) / units + 1, pieces = (units + G - 1) / G + 1;
    const int64_t w_cap = units * ((((a.T + kP - 1) / kP) + wph - 1) / wph);
    if (w_cap >= (int64_t{1} << 31) || G > kMaxBalancedCtas) return EXK_EARG;
    if (splits > ws->ns) return EXK_EARG;
    if (G * pieces > (int64_t{1} << 30)) return EXK_EARG;
    a.bal_G = static_cast<int>(G);
    a.bal_Su = 0;
    a.bal_W = 0;
    a.n_items = static_cast<int>(G * pieces);
    return 0;
  }
  const Balance b = balance_of(a.B, a.Hkv / hg, a.T, wph, sms);
  if (b.W >= (int64_t{1} << 31) || b.G > kMaxBalancedCtas) return EXK_EARG;
  if (b.splits > ws->ns) return EXK_EARG;  // the workspace must hold every piece of a unit
  if (b.G * b.pieces > (int64_t{1} << 30)) return EXK_EARG;
  a.bal_G = static_cast<int>(b.G);
  a.bal_Su = static_cast<int>(b.Su);
  a.bal_W = b.W;
  a.n_items = static_cast<int>(b.G * b.pieces);
  return 0;
}

}  // namespace

extern "C" int exk_plan_balanced(int B, int Hkv, int T, int num_ctas, int consumer_warps, int any_length,
                                 int32_t* ns_out) {
  if (B <= 0 || Hkv <= 0 || T <= 0 || num_ctas <= 0 || ns_out == nullptr) return EXK_EARG;
  if (consumer_warps != 4 && consumer_warps != 8) return EXK_EARG;
  const int hg = std::min(head_group(Hkv), consumer_warps);
  const int wph = consumer_warps / hg;
  const Balance b = balance_of(B, Hkv / hg, T, wph, num_ctas);
  // stages on the busiest CTA, each piece (item) costing ~2 stages of fixed
  // work (Q load, pipeline refill, epilogue), against the uniform plan's
  constexpr int64_t kItemOverhead = 2;
  const int64_t bal_cost = (b.W + b.G - 1) / b.G + kItemOverhead * b.pieces;
  int32_t ns = 0, sl = 0;
  const int64_t uni_cost = plan_for_heads(B, Hkv, T, num_ctas, hg, &ns, &sl);
  // any_length: the call reads one batch-wide length on the device (at most T):
  // the workspace bound that holds for every length
  const int64_t splits = any_length ? (b.G + b.units - 1) / b.units + 1 : b.splits;
  const bool fits = b.W < (int64_t{1} << 31) && b.G <= kMaxBalancedCtas;  // the kernel's exact quotients
  *ns_out = (fits && bal_cost < uni_cost && splits <= 4096) ? static_cast<int32_t>(splits) : 0;
  return 0;
}

namespace {

// A paged call (pages != nullptr) reads its pages from a pool of pool_pages
// pages through the block table; it needs one page per head per stage (the
// head group equal to the consumer warps), since consecutive pages of a
// sequence need not be adjacent in the pool.
int paged_args(AttnArgs& a, const int32_t* pages, int pages_stride, int pool_pages, int hg, int nwc) {
  if (pages == nullptr) return 0;
  if (pool_pages <= 0 || pages_stride < a.NP || hg != nwc) return EXK_EARG;
  if (static_cast<int64_t>(pool_pages) * kP * a.Hkv > (int64_t{1} << 31) - 1) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(pages) & 3u) != 0) return EXK_EALIGN;
  a.pages = pages;
  a.pages_stride = pages_stride;
  a.pool_pages = pool_pages;
  return 0;
}

int split_compressed(const uint16_t* q, const exk_cview* k, const exk_cview* v, int B, int TS, int Hkv, int Hq, int T,
                     int s0, int s1, const exk_partials* ws, int consumer_warps, float qk_scale, int32_t* status,
                     int device, void* stream, const int32_t* T_dev = nullptr, int T_add = 0, int T_stride = 0,
                     const int32_t* pages = nullptr, int pages_stride = 0, int pool_pages = 0) {
  if (k == nullptr || v == nullptr) return EXK_EARG;
  AttnArgs a;
  int r = common_args(a, q, B, TS, Hkv, Hq, T, s0, s1, ws, consumer_warps, qk_scale, status);
  if (r != 0) return r;
  a.T_dev = T_dev;
  a.T_add = T_add;
  a.T_stride = T_stride;
  const int hg = item_heads(ws, Hkv, consumer_warps);
  if ((r = paged_args(a, pages, pages_stride, pool_pages, hg, consumer_warps)) != 0) return r;
  int sms = 0;
  if ((r = use_device(device, &sms)) != 0) return r;
  const int wph = consumer_warps / hg;
  if ((r = balance_args(a, ws, hg, wph, sms)) != 0) return r;
  const exk_cview* cv[2] = {k, v};
  AttnMaps maps;
  const int64_t rows = pages ? static_cast<int64_t>(pool_pages) * kP : static_cast<int64_t>(B) * TS;
  const int64_t prows = rows / kP;
  for (int i = 0; i < 2; ++i) {
    const exk_cview* c = cv[i];
    if (!aligned16(c->sm) || !aligned16(c->code) || !aligned16(c->base) || !aligned16(c->raw)) return EXK_EALIGN;
    if (c->rowmask == nullptr || c->rowoff == nullptr || c->raw_rows <= 0) return EXK_EARG;
    a.rowmask[i] = c->rowmask;
    a.rowoff[i] = c->rowoff;
    a.raw[i] = c->raw;
    a.raw_rows[i] = c->raw_rows;
    if ((r = head_major_map(&maps.m[3 * i + 0], CU_TENSOR_MAP_DATA_TYPE_UINT8, c->sm, 128, 1, rows, Hkv, 128,
                            kP * wph, hg, CU_TENSOR_MAP_SWIZZLE_128B)) != 0)
      return r;
    if ((r = head_major_map(&maps.m[3 * i + 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, c->code, 64, 1, rows, Hkv, 64,
                            kP * wph, hg, CU_TENSOR_MAP_SWIZZLE_64B)) != 0)
      return r;
    if ((r = head_major_map(&maps.m[3 * i + 2], CU_TENSOR_MAP_DATA_TYPE_UINT8, c->base, 128, 1, prows, Hkv, 128,
                            wph, hg, CU_TENSOR_MAP_SWIZZLE_NONE)) != 0)
      return r;
  }
  const int grid = a.bal_G > 0 ? a.bal_G : static_cast<int>(std::min<int64_t>(a.n_items, sms));
  return dispatch_split<true>(a, maps, hg, grid, consumer_warps, device, static_cast<cudaStream_t>(stream));
}

int split_bf16(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int TS, int Hkv, int Hq, int T, int s0,
               int s1, const exk_partials* ws, int consumer_warps, float qk_scale, int32_t* status, int device,
               void* stream, const int32_t* T_dev = nullptr, int T_add = 0, int T_stride = 0,
               const int32_t* pages = nullptr, int pages_stride = 0, int pool_pages = 0) {
  if (k == nullptr || v == nullptr) return EXK_EARG;
  AttnArgs a;
  int r = common_args(a, q, B, TS, Hkv, Hq, T, s0, s1, ws, consumer_warps, qk_scale, status);
  if (r != 0) return r;
  a.T_dev = T_dev;
  a.T_add = T_add;
  a.T_stride = T_stride;
  const int hg = item_heads(ws, Hkv, consumer_warps);
  if ((r = paged_args(a, pages, pages_stride, pool_pages, hg, consumer_warps)) != 0) return r;
  int sms = 0;
  if ((r = use_device(device, &sms)) != 0) return r;
  if (!aligned16(k) || !aligned16(v)) return EXK_EALIGN;
  const int wph = consumer_warps / hg;
  if ((r = balance_args(a, ws, hg, wph, sms)) != 0) return r;
  AttnMaps maps;
  const int64_t rows = pages ? static_cast<int64_t>(pool_pages) * kP : static_cast<int64_t>(B) * TS;
  if ((r = head_major_map(&maps.m[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, k, 128, 2, rows, Hkv, 64, kP * wph, hg,
                          CU_TENSOR_MAP_SWIZZLE_128B)) != 0)
    return r;
  if ((r = head_major_map(&maps.m[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, v, 128, 2, rows, Hkv, 64, kP * wph, hg,
                          CU_TENSOR_MAP_SWIZZLE_128B)) != 0)
    return r;
  const int grid = a.bal_G > 0 ? a.bal_G : static_cast<int>(std::min<int64_t>(a.n_items, sms));
  return dispatch_split<false>(a, maps, hg, grid, consumer_warps, device, static_cast<cudaStream_t>(stream));
}

// Merge launch: a programmatic dependent of the preceding kernel on the stream
// (its CTAs are scheduled early and wait in griddepcontrol.wait).
int launch_merge(const exk_partials* ws, int rows, uint16_t* out, cudaStream_t stream, int32_t* advance = nullptr,
                 int n_adv = 0) {
  const bool wide = ws->ns > kWideSplits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(wide ? rows : (rows + 3) / 4);
  cfg.blockDim = dim3(wide ? wide_warps(ws->ns) * 32 : 128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, wide ? merge_kernel<true> : merge_kernel<false>,
                                           static_cast<const float*>(ws->o),
                                           static_cast<const float*>(ws->m), static_cast<const float*>(ws->l), ws->ns,
                                           rows, out, advance, n_adv);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

}  // namespace

extern "C" int exk_attn_split_compressed(const uint16_t* q, const exk_cview* k, const exk_cview* v, int B, int TS,
                                         int Hkv, int Hq, int T, int s0, int s1, const exk_partials* ws,
                                         int consumer_warps, float qk_scale, int32_t* status, int device,
                                         void* stream) {
  return split_compressed(q, k, v, B, TS, Hkv, Hq, T, s0, s1, ws, consumer_warps, qk_scale, status, device, stream);
}

extern "C" int exk_attn_split_bf16(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int TS, int Hkv,
                                   int Hq, int T, int s0, int s1, const exk_partials* ws, int consumer_warps,
                                   float qk_scale, int32_t* status, int device, void* stream) {
  return split_bf16(q, k, v, B, TS, Hkv, Hq, T, s0, s1, ws, consumer_warps, qk_scale, status, device, stream);
}

extern "C" int exk_attention_compressed(const uint16_t* q, const exk_cview* k, const exk_cview* v, int B, int TS,
                                        int Hkv, int Hq, int T, const exk_partials* ws, uint16_t* out,
                                        int consumer_warps, float qk_scale, int32_t* status, int device,
                                        void* stream) {
  if (ws == nullptr || out == nullptr) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  int r = split_compressed(q, k, v, B, TS, Hkv, Hq, T, 0, ws->ns, ws, consumer_warps, qk_scale, status, device,
                           stream);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream));
}

// Checks shared by the device-length entries.
int devlen_args(const exk_partials* ws, const uint16_t* out, const int32_t* T_dev, int T_cap, int T_stride,
                int advance) {
  if (ws == nullptr || out == nullptr || T_dev == nullptr || (T_stride != 0 && T_stride != 1)) return EXK_EARG;
  if (advance != 0 && T_stride != 0) return EXK_EARG;  // only a batch-wide length is advanced by the merge
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0 || (reinterpret_cast<uintptr_t>(T_dev) & 3u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  const int last = (T_cap - 1) / (ws->split_len > 0 ? ws->split_len : 1);
  if (T_cap <= 0 || (ws->split_len != 0 && last + 1 != ws->ns)) return EXK_EARG;  // the plan must be the capacity's
  return 0;
}

extern "C" int exk_attention_compressed_devlen(const uint16_t* q, const exk_cview* k, const exk_cview* v, int B,
                                               int TS, int Hkv, int Hq, int T_cap, int32_t* T_dev, int T_add,
                                               int T_stride, int advance, const exk_partials* ws, uint16_t* out,
                                               int consumer_warps, float qk_scale, int32_t* status, int device,
                                               void* stream) {
  int r = devlen_args(ws, out, T_dev, T_cap, T_stride, advance);
  if (r != 0) return r;
  r = split_compressed(q, k, v, B, TS, Hkv, Hq, T_cap, 0, ws->ns, ws, consumer_warps, qk_scale, status, device,
                       stream, T_dev, T_add, T_stride);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream), advance ? T_dev : nullptr,
                                   advance);
}

extern "C" int exk_attention_compressed_paged(const uint16_t* q, const exk_cview* k, const exk_cview* v,
                                              int pool_pages, int Hkv, int B, int Hq, const int32_t* block_table,
                                              int max_pages, const int32_t* seq_lens, const exk_partials* ws,
                                              uint16_t* out, int consumer_warps, float qk_scale, int32_t* status,
                                              int device, void* stream) {
  if (block_table == nullptr || max_pages <= 0 || max_pages > (1 << 26)) return EXK_EARG;
  const int T_cap = max_pages * kP;
  int r = devlen_args(ws, out, seq_lens, T_cap, 1, 0);
  if (r != 0) return r;
  r = split_compressed(q, k, v, B, T_cap, Hkv, Hq, T_cap, 0, ws->ns, ws, consumer_warps, qk_scale, status, device,
                       stream, seq_lens, 0, 1, block_table, max_pages, pool_pages);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream));
}

extern "C" int exk_attention_bf16_paged(const uint16_t* q, const uint16_t* k, const uint16_t* v, int pool_pages,
                                        int Hkv, int B, int Hq, const int32_t* block_table, int max_pages,
                                        const int32_t* seq_lens, const exk_partials* ws, uint16_t* out,
                                        int consumer_warps, float qk_scale, int32_t* status, int device,
                                        void* stream) {
  if (block_table == nullptr || max_pages <= 0 || max_pages > (1 << 26)) return EXK_EARG;
  const int T_cap = max_pages * kP;
  int r = devlen_args(ws, out, seq_lens, T_cap, 1, 0);
  if (r != 0) return r;
  r = split_bf16(q, k, v, B, T_cap, Hkv, Hq, T_cap, 0, ws->ns, ws, consumer_warps, qk_scale, status, device, stream,
                 seq_lens, 0, 1, block_table, max_pages, pool_pages);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream));
}

extern "C" int exk_attention_bf16_devlen(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int TS,
                                         int Hkv, int Hq, int T_cap, int32_t* T_dev, int T_add, int T_stride,
                                         int advance, const exk_partials* ws, uint16_t* out, int consumer_warps,
                                         float qk_scale, int32_t* status, int device, void* stream) {
  int r = devlen_args(ws, out, T_dev, T_cap, T_stride, advance);
  if (r != 0) return r;
  r = split_bf16(q, k, v, B, TS, Hkv, Hq, T_cap, 0, ws->ns, ws, consumer_warps, qk_scale, status, device, stream,
                 T_dev, T_add, T_stride);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream), advance ? T_dev : nullptr,
                                   advance);
}

extern "C" int exk_attention_bf16(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int TS, int Hkv,
                                  int Hq, int T, const exk_partials* ws, uint16_t* out, int consumer_warps,
                                  float qk_scale, int32_t* status, int device, void* stream) {
  if (ws == nullptr || out == nullptr) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  int r = split_bf16(q, k, v, B, TS, Hkv, Hq, T, 0, ws->ns, ws, consumer_warps, qk_scale, status, device, stream);
  return r != 0 ? r : launch_merge(ws, B * Hq, out, static_cast<cudaStream_t>(stream));
}

extern "C" int exk_attn_merge(const exk_partials* ws, int rows, uint16_t* out, int device, void* stream) {
  if (ws == nullptr || out == nullptr || rows <= 0 || ws->ns <= 0) return EXK_EARG;
  if (!aligned16(ws->o) || (reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  return launch_merge(ws, rows, out, static_cast<cudaStream_t>(stream));
}

namespace {

// Fills the split layout of a gathered or peer merge; 0 or an EXK_E* code.
int gather_layout(GatherArgs& g, int world, const int32_t* counts, int nmax, int rows) {
  if (counts == nullptr || world <= 0 || world > kMaxRanks || nmax <= 0 || rows <= 0) return EXK_EARG;
  g.rows = rows;
  g.nmax = nmax;
  g.world = world;
  g.pre[0] = 0;
  for (int r = 0; r < world; ++r) {
    if (counts[r] < 0 || counts[r] > nmax) return EXK_EARG;
    g.pre[r + 1] = g.pre[r] + counts[r];
  }
  for (int r = world + 1; r <= kMaxRanks; ++r) g.pre[r] = g.pre[world];
  g.ns = g.pre[world];
  return g.ns > 0 ? 0 : EXK_EARG;
}

// Launched as a programmatic dependent of the preceding kernel on the stream,
// like the single-GPU merge.
int launch_gathered(const GatherArgs& g, uint16_t* out, int device, void* stream) {
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  const bool wide = g.ns > kWideSplits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(wide ? g.rows : (g.rows + 3) / 4);
  cfg.blockDim = dim3(wide ? wide_warps(g.ns) * 32 : 128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, wide ? merge_gathered_kernel<true> : merge_gathered_kernel<false>, g, out);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

}  // namespace

extern "C" int exk_attn_merge_partial(const exk_partials* ws, int rows, int s0, int s1, float* o, float* m, float* l,
                                      int device, void* stream) {
  if (ws == nullptr || o == nullptr || m == nullptr || l == nullptr || rows <= 0) return EXK_EARG;
  if (s0 < 0 || s1 > ws->ns || s0 >= s1) return EXK_EARG;
  if (!aligned16(ws->o) || !aligned16(o)) return EXK_EALIGN;
  int r = use_device(device, nullptr);
  if (r != 0) return r;
  const int n = s1 - s0;
  const bool wide = n > kWideSplits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(wide ? rows : (rows + 3) / 4);
  cfg.blockDim = dim3(wide ? wide_warps(n) * 32 : 128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, wide ? merge_partial_kernel<true> : merge_partial_kernel<false>,
                                           static_cast<const float*>(ws->o), static_cast<const float*>(ws->m),
                                           static_cast<const float*>(ws->l), static_cast<int>(ws->ns), s0, n, rows, o,
                                           m, l);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int exk_attn_merge_gathered(const float* buf, int world, const int32_t* counts, int nmax, int rows,
                                       uint16_t* out, int device, void* stream) {
  if (buf == nullptr || out == nullptr) return EXK_EARG;
  if (!aligned16(buf) || (reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  GatherArgs g = {};
  int r = gather_layout(g, world, counts, nmax, rows);
  if (r != 0) return r;
  const int64_t block = (static_cast<int64_t>(rows) * nmax * (kD + 2) + 3) & ~int64_t{3};
  for (int i = 0; i < world; ++i) g.base[i] = buf + i * block;
  return launch_gathered(g, out, device, stream);
}

extern "C" int exk_attn_merge_peers(const float* const* blocks, int world, int rank, const int32_t* counts, int nmax,
                                    int rows, uint32_t* flags, uint32_t* const* peer_flags, uint32_t epoch,
                                    uint16_t* out, int32_t* status, int device, void* stream) {
  if (blocks == nullptr || out == nullptr || rank < 0 || rank >= world) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (device_reachable(out) != 0) return EXK_EARG;
  GatherArgs g = {};
  int r = gather_layout(g, world, counts, nmax, rows);
  if (r != 0) return r;
  for (int i = 0; i < world; ++i) {
    if (blocks[i] == nullptr) return EXK_EARG;
    if (!aligned16(blocks[i])) return EXK_EALIGN;
    g.base[i] = blocks[i];
  }
  if (world > 1) {
    if (flags == nullptr || peer_flags == nullptr || (reinterpret_cast<uintptr_t>(flags) & 3u) != 0) return EXK_EARG;
    for (int i = 0; i < world; ++i) {
      if (i != rank && (peer_flags[i] == nullptr || (reinterpret_cast<uintptr_t>(peer_flags[i]) & 3u) != 0))
        return EXK_EARG;
      g.peer_flag[i] = peer_flags[i];
    }
    g.flags = flags;
  }
  g.epoch = epoch;
  g.rank = rank;
  g.status = status;
  return launch_gathered(g, out, device, stream);
}
