// clefq: tensor-parallel dense MLP helpers (the intermediate dimension sharded over GPUs).
//
// The reference runs the MLP block (src/backbone.rs:880-894, src/quantized.rs:406-439) on one
// GPU.  Sharded over G ranks, rank r owns intermediate rows [r*I/G, (r+1)*I/G) of gate and up
// and output rows [r*H/G, (r+1)*H/G) of down:
//
//   packed x (replicated) -> gate|up shard -> SwiGLU shard row maxima -> all-reduce(max)
//   -> pack the shard with the full-row maxima -> all-gather packed codes -> unpack into the
//   full s8 operand -> down shard -> all-gather output columns -> interleave
//
// Hadamard groups never straddle shards (I/G is a multiple of 256), every row scale is taken
// from the maximum over the whole row, and every GEMM output column sees the full K, so the
// result is bit-identical to one GPU.
#include "cq_common.cuh"
#include "clefq_internal.h"

namespace cq {

// codes [G][rows][shard_words] (int4 words, the shards of each row in rank order) ->
// s8 operand [rows][G * shard_words * 8]: 16 * code, low nibbles of every 4-word group first.
__global__ void tp_gather_unpack_kernel(const uint32_t *__restrict__ codes, int world, int64_t rows, int shard_words,
                                        uint8_t *__restrict__ op, int64_t op_ld) {
  const int groups_per_shard = shard_words / 4;
  const int64_t per_row = (int64_t)world * groups_per_shard;
  const int64_t total = rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / per_row;
    const int64_t gq = i % per_row;  // 4-word group index along the full row
    const int g = (int)(gq / groups_per_shard);
    const int local = (int)(gq % groups_per_shard);
    const uint4 v = *reinterpret_cast<const uint4 *>(codes + ((int64_t)g * rows + m) * shard_words + local * 4);
    uint4 *dst = reinterpret_cast<uint4 *>(op + m * op_ld + gq * 32);
    dst[0] = make_uint4(nib_lo16(v.x), nib_lo16(v.y), nib_lo16(v.z), nib_lo16(v.w));
    dst[1] = make_uint4(nib_hi16(v.x), nib_hi16(v.y), nib_hi16(v.z), nib_hi16(v.w));
  }
}

int launch_tp_gather_unpack(const uint32_t *codes, int world, int64_t rows, int shard_words, uint8_t *op,
                            int64_t op_ld, cudaStream_t stream, int num_sms) {
  const int64_t total = rows * world * (shard_words / 4);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  tp_gather_unpack_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(codes, world, rows,
                                                                                       shard_words, op, op_ld);
  return launch_check();
}

// src [G][rows][shard_bytes] -> dst [rows][dst_ld]: dst[m][g*shard_bytes + j] = src[g][m][j],
// 16 bytes per thread.
__global__ void tp_interleave_kernel(const uint8_t *__restrict__ src, int world, int64_t rows, int64_t shard_bytes,
                                     uint8_t *__restrict__ dst, int64_t dst_ld) {
  const int64_t chunks = shard_bytes / 16;
  const int64_t per_row = world * chunks;
  const int64_t total = rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / per_row;
    const int64_t c = i % per_row;
    const int64_t g = c / chunks, j = c % chunks;
    *reinterpret_cast<uint4 *>(dst + m * dst_ld + c * 16) =
        *reinterpret_cast<const uint4 *>(src + (g * rows + m) * shard_bytes + j * 16);
  }
}

int launch_tp_interleave(const uint8_t *src, int world, int64_t rows, int64_t shard_bytes, uint8_t *dst,
                         int64_t dst_ld, cudaStream_t stream, int num_sms) {
  const int64_t total = rows * world * (shard_bytes / 16);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  tp_interleave_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(src, world, rows, shard_bytes, dst,
                                                                                    dst_ld);
  return launch_check();
}

}  // namespace cq
