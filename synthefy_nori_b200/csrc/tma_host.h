// Host-side TMA descriptor construction. The driver entry point
// cuTensorMapEncodeTiled is resolved once through the runtime
// (cudaGetDriverEntryPoint), so the extension does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <array>
#include <mutex>
#include <vector>

namespace nori {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D bf16 tensor [rows, cols] with row stride `ld` elements; box = box_cols x box_rows,
// 128-byte swizzle (box_cols * 2 must be 128). Out-of-bounds elements read as zero.
inline CUtensorMap make_tmap_2d_bf16(void* base, int64_t cols, int64_t rows, int64_t ld, int box_cols, int box_rows,
                                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return m;
}

}  // namespace nori

namespace nori {

// Up-to-5-D tensor map (bf16 unless `dtype` says otherwise): dims[0] is the contiguous
// dimension; strides_bytes[i] is the byte stride of dims[i + 1]; box[i] elements per
// dimension; 128B swizzle.
inline CUtensorMap make_tmap_nd_bf16(void* base, int rank, const int64_t* dims, const int64_t* strides_bytes,
                                     const int* box, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
                                     CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(rank >= 1 && rank <= 5, "TMA rank 1..5");
  CUtensorMap m;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    b[i] = static_cast<cuuint32_t>(box[i]);
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    TORCH_CHECK(strides_bytes[i] % 16 == 0, "TMA strides must be multiples of 16 bytes");
    s[i] = static_cast<cuuint64_t>(strides_bytes[i]);
  }
  CUresult r = encode_tiled_fn()(&m, dtype, rank, base, d, s, b, e,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (rank ", rank, ") failed with code ", static_cast<int>(r));
  return m;
}

// A strided [.., rows, d] view given as the layout (s0, s1, s2, row, d1, d2) (element
// strides of the i0 / i1 / i2 / row indices; bh -> (i0, i1, i2) with i2 fastest) -> 5-D map
// with the non-contiguous dimensions sorted by stride. The box is box_cols x 1 x .. x
// box_rows rows x ..; the contiguous dimension has extent d_valid, so columns past it (head
// padding) and rows past n_rows read as zero.
struct Map5 {
  CUtensorMap map;
  int pos[4];  // positions of row, i2, i1, i0
};

inline Map5 make_map(const torch::Tensor& t, const std::vector<int64_t>& l, int64_t n_rows, int64_t n_i0, int d_valid,
              int elem_bytes = 2, int box_cols = 64, int box_rows = 128,
              CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  struct Dim {
    int64_t extent, stride;
    int role;  // 0 row, 1 i2, 2 i1, 3 i0
  };
  const int64_t d1 = l[4], d2 = l[5];
  std::array<Dim, 4> dims = {Dim{n_rows, l[3], 0}, Dim{d2, l[2], 1}, Dim{d1, l[1], 2}, Dim{n_i0, l[0], 3}};
  // dimensions of extent 1 get a harmless stride (never stepped)
  int64_t big = 1;
  for (auto& d : dims) big = std::max(big, d.stride * std::max<int64_t>(d.extent, 1));
  for (auto& d : dims)
    if (d.extent <= 1 || d.stride == 0) d.stride = big;
  std::stable_sort(dims.begin(), dims.end(), [](const Dim& a, const Dim& b) { return a.stride < b.stride; });
  int64_t ext[5], strides[4];
  int box[5];
  ext[0] = d_valid;
  box[0] = box_cols;
  Map5 m{};
  for (int i = 0; i < 4; ++i) {
    ext[i + 1] = std::max<int64_t>(dims[i].extent, 1);
    strides[i] = dims[i].stride * elem_bytes;
    box[i + 1] = dims[i].role == 0 ? box_rows : 1;
    m.pos[dims[i].role] = i + 1;
  }
  m.map = make_tmap_nd_bf16(t.data_ptr(), 5, ext, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, dtype);
  return m;
}

// SMs kept free of the persistent (one CTA per SM) kernels while gradient-communication
// kernels run beside them on other streams: a persistent grid that covers every SM would
// otherwise have a CTA waiting for an SM held by a communication kernel (which may itself
// be waiting for a peer), stretching the whole kernel. Set by the multi-GPU data-parallel
// path; 0 (every SM) otherwise.
int sm_reserve();
void set_sm_reserve(int64_t n);
inline int persistent_sms(int n_sm) { return std::max(1, n_sm - sm_reserve()); }

}  // namespace nori
