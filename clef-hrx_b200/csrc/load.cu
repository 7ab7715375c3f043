// clefq: the weight-load path (src/quantized.rs:147-234): BF16 checkpoint rows -> per-row
// Hadamard-rotated int4/int8 codes -> 128 x 32-word tiles plus the compact f32 scale row.
//
// Checkpoint projections may be stored in the tiled GEMM layout of src/checkpoint.rs:20-100,
// "tiled256x64": a [rows][cols] BF16 matrix as [rows/256][cols/64][256][64].  The reference
// restores row-major order on the host before uploading; here the tiled bytes are uploaded
// as they are and one kernel permutes them on the device.
#include "cq_common.cuh"
#include "clefq_internal.h"

namespace cq {

constexpr int64_t kTileRows = 256, kTileCols = 64;

// dst row-major [rows][cols] <- src tiled; one 16-byte vector (8 BF16 of one 64-column
// segment) per thread, consecutive threads on consecutive destination vectors.
__global__ void untile_kernel(const uint4 *__restrict__ src, int64_t rows, int64_t cols, uint4 *__restrict__ dst) {
  const int64_t vec_per_row = cols / 8;
  const int64_t total = rows * vec_per_row;
  const int64_t k_tiles = cols / kTileCols;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = v / vec_per_row;
    const int64_t k = (v % vec_per_row) * 8;
    const int64_t pos = (((n / kTileRows) * k_tiles + k / kTileCols) * kTileRows + n % kTileRows) * kTileCols +
                        k % kTileCols;
    dst[v] = src[pos / 8];
  }
}

int launch_untile(const uint16_t *src, int64_t rows, int64_t cols, uint16_t *dst, cudaStream_t stream, int num_sms) {
  const int64_t total = rows * cols / 8;
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  untile_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(
      reinterpret_cast<const uint4 *>(src), rows, cols, reinterpret_cast<uint4 *>(dst));
  return launch_check();
}

namespace {
int64_t weight_stride(int64_t cols, int bits) { return cols + (cols % 1024 == 0 ? 512 / bits : 0); }

Arena load_tables(Arena a, int64_t rows, int64_t cols, int bits, bool tiled, uint16_t **dense, uint32_t **packed) {
  *dense = tiled ? a.take<uint16_t>(rows * cols) : nullptr;
  *packed = a.take<uint32_t>(rows * (weight_stride(cols, bits) / (32 / bits) + 1));
  return a;
}

bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }
}  // namespace

}  // namespace cq

using namespace cq;

extern "C" {

int clefq_untile_bf16(void *stream, const void *src, int64_t rows, int64_t cols, void *dst) {
  if (rows <= 0 || cols <= 0 || rows % kTileRows || cols % kTileCols)
    return report_error(CLEFQ_ERR_SHAPE, "tiled layout requires 256-row and 64-column multiples");
  if (!al16(src) || !al16(dst)) return report_error(CLEFQ_ERR_ALIGN, "untile buffers must be 16-byte aligned");
  const int rc = launch_untile(static_cast<const uint16_t *>(src), rows, cols, static_cast<uint16_t *>(dst),
                               static_cast<cudaStream_t>(stream), device_sms());
  return rc ? report_error(rc, "untile launch failed") : 0;
}

int64_t clefq_load_weight_workspace_size(int64_t rows, int64_t cols, int bits, int tiled) {
  if (rows <= 0 || cols <= 0 || !(bits == 4 || bits == 8)) return -1;
  uint16_t *d;
  uint32_t *p;
  return aligned_total(load_tables(Arena{nullptr, INT64_MAX}, rows, cols, bits, tiled != 0, &d, &p));
}

int clefq_load_weight(void *stream, const void *src, int64_t rows, int64_t cols, int bits, int tiled,
                      void *codes_tiled, float *scales, void *workspace, int64_t workspace_bytes) {
  if (!(bits == 4 || bits == 8)) return report_error(CLEFQ_ERR_SHAPE, "unsupported rotated integer operand");
  if (rows <= 0 || cols <= 0 || rows % 256 || cols % 256)
    return report_error(CLEFQ_ERR_SHAPE, "unsupported quantized weight shape");
  if (!src || !codes_tiled || !scales) return report_error(CLEFQ_ERR_SHAPE, "load weight: null buffer");
  uint16_t *dense;
  uint32_t *packed;
  Arena a = load_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, rows, cols, bits, tiled != 0,
                        &dense, &packed);
  if (!a.ok || !workspace) return report_error(CLEFQ_ERR_WORKSPACE, "load weight workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void *rows_src = src;
  if (tiled) {
    int rc = clefq_untile_bf16(stream, src, rows, cols, dense);
    if (rc) return rc;
    rows_src = dense;
  }
  const int64_t stride = weight_stride(cols, bits);
  const int64_t words = stride / (32 / bits);
  // weights rotate and quantise like activations, then move to 128 x 32-word tiles
  int rc = clefq_prepare(stream, CLEFQ_PREP_PLAIN, bits, rows_src, cols, nullptr, 0, rows, cols, stride, packed,
                         nullptr, 0, nullptr, 0);
  if (rc) return rc;
  rc = clefq_retile(stream, packed, rows, cols, bits, words, codes_tiled);
  if (rc) return rc;
  if (cudaMemcpyAsync(scales, packed + rows * words, rows * sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return report_error(CLEFQ_ERR_CUDA, "load weight: scale copy");
  return 0;
}

}  // extern "C"
