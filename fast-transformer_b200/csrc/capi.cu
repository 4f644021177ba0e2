// Library-wide pieces of the C ABI: version, the device error word, the tensor-map
// encoder (fetched from the driver at run time, so the library needs no -lcuda), and
// device-property caching.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace fb {

__device__ unsigned g_error_word = 0;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encoder() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult status;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &status) ==
          cudaSuccess &&
      status == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
unsigned* g_error_ptr[kMaxDevices] = {nullptr};

}  // namespace

int encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                   uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  std::call_once(g_encode_once, load_encoder);
  if (g_encode == nullptr) return FB_ERR_DRIVER;
  // The TMA unit wants a 16-byte aligned base and 16-byte multiple pitches.
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch_elems * 2) % 16 != 0)
    return FB_ERR_ARG;
  if (rows == 0 || cols == 0 || rows > (1ull << 32) || cols > (1ull << 32)) return FB_ERR_SHAPE;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FB_OK : FB_ERR_DRIVER;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < kMaxDevices && g_sm_count[dev] > 0) return g_sm_count[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev >= 0 && dev < kMaxDevices) g_sm_count[dev] = n;
  return n;
}

unsigned* error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_error_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    g_error_ptr[dev] = static_cast<unsigned*>(p);
  }
  return g_error_ptr[dev];
}

int check_launch() { return cudaGetLastError() == cudaSuccess ? FB_OK : FB_ERR_LAUNCH; }

}  // namespace fb

extern "C" int fb_version(void) { return 1; }

extern "C" int fb_device_error(unsigned int* host_flags) {
  if (host_flags == nullptr) return FB_ERR_ARG;
  unsigned zero = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return FB_ERR_LAUNCH;
  if (cudaMemcpyFromSymbol(host_flags, fb::g_error_word, sizeof(unsigned)) != cudaSuccess)
    return FB_ERR_LAUNCH;
  if (cudaMemcpyToSymbol(fb::g_error_word, &zero, sizeof(unsigned)) != cudaSuccess)
    return FB_ERR_LAUNCH;
  return FB_OK;
}
