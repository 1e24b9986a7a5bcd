// tma_maps.cu: TMA tensor-map encoding for [B, H, N, D] operands, shared by
// the tensor-core kernels. cuTensorMapEncodeTiled is a driver entry point,
// fetched once through the runtime (no link-time dependency on libcuda).
#include <mutex>

#include "rbf_common.cuh"

namespace vectra {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

bool tensor_maps_available() { return encode_fn() != nullptr; }

bool make_tile_map(CUtensorMap* map, const void* base, int dtype, int64_t B,
                   int64_t H, int64_t N, int64_t D, const int64_t* s,
                   int box_rows, int box_cols) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int64_t es = 2;
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(H),
                        cuuint64_t(B)};
  cuuint64_t strides[3] = {cuuint64_t(s[2] * es), cuuint64_t(s[1] * es),
                           cuuint64_t(s[0] * es)};
  // Strides of size-1 dimensions are never used; give them valid values.
  if (N == 1) strides[0] = cuuint64_t(D * es + 15) / 16 * 16;
  if (H == 1) strides[1] = strides[0] * N;
  if (B == 1) strides[2] = strides[1] * H;
  // The swizzle span is the box's row: 128, 64 or 32 bytes.
  const int row_bytes = box_cols * int(es);
  if (row_bytes != 128 && row_bytes != 64 && row_bytes != 32) return false;
  const CUtensorMapSwizzle swizzle =
      row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                       : (row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : CU_TENSOR_MAP_SWIZZLE_32B);
  cuuint32_t box[4] = {cuuint32_t(box_cols), cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map,
                        dtype == VECTRA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace vectra
