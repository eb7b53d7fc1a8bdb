// Device queries cached per device.
#include <mutex>
#include <set>
#include <utility>

#include <cudaTypedefs.h>

#include "internal.h"

namespace rwkvb {

int device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

int allow_big_smem(const void* kernel) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, kernel})) return RWKVB_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
  if (e != cudaSuccess) return cuda_status(e);
  done.insert({dev, kernel});
  return RWKVB_OK;
}

int encode_u8_map(CUtensorMap* out, int rank, const void* addr, const uint64_t* dims, const uint64_t* strides,
                  const uint32_t* box, bool swizzle128) {
  static std::mutex mu;
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || !p) {
        cudaGetLastError();
        return RWKVB_EUNSUPPORTED;
      }
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
    }
  }
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(addr), d, st, b, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RWKVB_OK : RWKVB_EUNSUPPORTED;
}

}  // namespace rwkvb
