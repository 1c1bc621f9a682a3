// Host utilities and error strings of the C ABI.
#include <mutex>

#include "../../include/exactkv_b200.h"
#include "exk_host.h"

namespace exk {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

constexpr int kMaxDevices = 64;
int g_num_sms[kMaxDevices] = {};

}  // namespace

int make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                 uint32_t box2, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return EXK_EDRIVER;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, box2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : EXK_ETMAP;
}

int use_device(int device, int* num_sms) {
  if (device < 0 || device >= kMaxDevices) return EXK_EARG;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (g_num_sms[device] == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_num_sms[device] = n;
  }
  if (num_sms != nullptr) *num_sms = g_num_sms[device];
  return 0;
}

int device_reachable(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error this call may leave
    return EXK_EARG;
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return 0;
  if (at.type == cudaMemoryTypeHost && at.devicePointer == p) return 0;
  return EXK_EARG;
}

}  // namespace exk

extern "C" int exk_num_sms(int device) {
  int n = 0;
  int r = exk::use_device(device, &n);
  return r == 0 ? n : r;
}

extern "C" const char* exk_error_string(int code) {
  switch (code) {
    case 0: return "ok";
    case EXK_EARG: return "exactkv_b200: shape or count out of range";
    case EXK_EALIGN: return "exactkv_b200: pointer or stride not 16-byte aligned";
    case EXK_ETMAP: return "exactkv_b200: cuTensorMapEncodeTiled rejected a tensor map";
    case EXK_EDRIVER: return "exactkv_b200: cuTensorMapEncodeTiled entry point unavailable";
    case EXK_EHEADS: return "exactkv_b200: more than 16 query heads per KV head";
    case EXK_ESCRATCH: return "exactkv_b200: split partials exceed the fixed scratch of exk_attention_compressed_noalloc";
    default: break;
  }
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "exactkv_b200: unknown error";
}

extern "C" const char* exk_status_string(int code) {
  switch (code) {
    case EXK_S_OK: return "ok";
    case EXK_S_FULL_TIMEOUT: return "attention consumer waited more than 2 s for a staged page";
    case EXK_S_EMPTY_TIMEOUT: return "TMA producer waited more than 2 s for a free ring slot";
    case EXK_S_RAW_INDEX: return "rowoff/rowmask point past the end of the raw pool";
    case EXK_S_CHAIN_TIMEOUT: return "encoder CTA waited more than 2 s for its predecessor's offset";
    case EXK_S_DRAIN_TIMEOUT: return "in-flight TMA copies did not land within 2 s";
    case EXK_S_PEER_TIMEOUT: return "peer merge waited more than 2 s for another GPU's signal";
    case EXK_S_PAGE_INDEX: return "a block-table entry names a page outside the pool (read as zeros)";
    default: return "unknown device status";
  }
}
