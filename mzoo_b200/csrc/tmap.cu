// Host helper: build a TMA tensor map with cuTensorMapEncodeTiled, reached through the
// CUDA runtime's driver entry point so the library does not link libcuda directly.
#include "tc.cuh"

namespace mzb {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  MZB_REQUIRE(fn != nullptr, MZB_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable (driver too old?)");
  MZB_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0, MZB_ERR_ALIGN, "TMA base pointer not 16-byte aligned");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i < rank - 1) {
      s[i] = strides_bytes[i];
      MZB_REQUIRE(s[i] % 16 == 0, MZB_ERR_ALIGN, "TMA stride %llu not a multiple of 16 bytes",
                  (unsigned long long)s[i]);
    }
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    // a host thread whose first CUDA call this is (e.g. the autograd engine's backward
    // thread) has no current context yet: bind the current device's primary context and retry
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess)
      r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  MZB_REQUIRE(r == CUDA_SUCCESS, MZB_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return MZB_OK;
}

}  // namespace mzb
