// Compressed decode attention that allocates nothing: the split-K partials live
// in a fixed array inside this library instead of a caller-provided workspace.
//
// Who needs it: a host that cannot allocate device memory at call time — a
// serving runtime that plans all device memory up front, or a plugin whose
// enqueue step must not call cudaMalloc (which may synchronise the device or
// be forbidden there) — and has no workspace of its own to pass in. It passes
// only q, the two caches and the output.
//
// The cost: EXK_NOALLOC_SCRATCH_BYTES of device memory, held by every GPU that
// loads this library until the process exits, and one shared scratch area per
// GPU, so calls that overlap on the GPU (for example on two streams) race.
#include <mutex>

#include "../../include/exactkv_b200.h"
#include "exk_host.h"

namespace exk {
namespace {

// Split partials of one call: o [rows, ns, 128], then m [rows, ns], then l [rows, ns] (fp32).
static __device__ __align__(256) float g_partials[EXK_NOALLOC_SCRATCH_BYTES / sizeof(float)];

constexpr int kMaxDev = 64;
std::mutex g_mu;
float* g_dev_ptr[kMaxDev] = {};

// The array's name is a host-side stand-in in host code; the kernels need its
// device address, looked up once per device with that device current. The
// address is cached for the life of the process and not looked up again after
// a cudaDeviceReset (the library's other entry points do not survive a reset
// of their caller's context either).
int scratch_address(int device, float** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_dev_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_partials);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_dev_ptr[device] = static_cast<float*>(p);
  }
  *out = g_dev_ptr[device];
  return 0;
}

}  // namespace
}  // namespace exk

extern "C" int exk_attention_compressed_noalloc(const uint16_t* q, const exk_cview* k, const exk_cview* v, int B,
                                                int TS, int Hkv, int Hq, int T, int consumer_warps, float qk_scale,
                                                uint16_t* out, int32_t* status, int device, void* stream) {
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || T <= 0 || device < 0 || device >= exk::kMaxDev) return EXK_EARG;
  // The shape and output checks of the allocating entry points, before the
  // scratch size is computed: a bad shape reports its own error (not
  // EXK_ESCRATCH), and nothing is launched when any argument is refused.
  if (TS <= 0 || TS % EXK_PAGE != 0 || T > TS || Hq % Hkv != 0) return EXK_EARG;
  if (Hq / Hkv > 16) return EXK_EHEADS;
  if (out == nullptr || q == nullptr || k == nullptr || v == nullptr) return EXK_EARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return EXK_EALIGN;
  if (exk::device_reachable(out) != 0) return EXK_EARG;
  int sms = 0;
  int r = exk::use_device(device, &sms);  // makes `device` current before the symbol lookup
  if (r != 0) return r;
  int32_t ns = 0, split_len = 0;
  if ((r = exk_plan_splits(B, Hkv, T, sms, &ns, &split_len)) != 0) return r;
  const int64_t rows = static_cast<int64_t>(B) * Hq;
  const int64_t need = rows * ns * (EXK_HEAD_DIM + 2) * static_cast<int64_t>(sizeof(float));
  if (need > static_cast<int64_t>(EXK_NOALLOC_SCRATCH_BYTES)) return EXK_ESCRATCH;
  float* base = nullptr;
  if ((r = exk::scratch_address(device, &base)) != 0) return r;
  // Every partial the merge reads is written by this call's split kernel first,
  // so the previous call's leftovers need no clearing.
  exk_partials ws;
  ws.o = base;
  ws.m = base + rows * ns * EXK_HEAD_DIM;
  ws.l = ws.m + rows * ns;
  ws.ns = ns;
  ws.split_len = split_len;
  ws.heads = 0;
  if ((r = exk_attn_split_compressed(q, k, v, B, TS, Hkv, Hq, T, 0, ns, &ws, consumer_warps, qk_scale, status,
                                     device, stream)) != 0)
    return r;
  return exk_attn_merge(&ws, static_cast<int>(rows), out, device, stream);
}
