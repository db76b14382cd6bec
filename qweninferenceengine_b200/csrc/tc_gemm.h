// tc_gemm.h -- batched projections on the 5th-generation tensor cores
// (tcgen05.mma, fp16 operands, fp32 accumulators in tensor memory).
//
// One launch computes Y[b][n] = sum_k W[n][k] * X[b][k] for up to 256 rows b
// of activations: the Q4 block-32 projections of gemv_q4_0 (matmul.metal:9-73)
// with the weights dequantised to fp16 on the fly, and the fp16 LM head of
// gemv_fp16 (matmul.metal:75-113), for many sequences at once.
//
// Layouts (all written by this library; none is the reference's file layout):
//   Q4 weight blob   [n/128 tiles][k/64 chunks] x 4608 B:
//                      [2 halves][128 rows][16 B]  packed nibbles of block
//                                                  2c+h of each row, every
//                                                  32-bit word nibble-permuted
//                                                  (nibble s = k_2s, nibble
//                                                  4+s = k_2s+1)
//                      [128 rows][2] fp16          the two block scales
//   fp16 weight blob [n/128 tiles][k/64 chunks] x 16384 B: 128 rows x 128 B,
//                      16-byte chunk j of row r at (j ^ (r & 7)) -- the
//                      tensor core's 128-byte-swizzled K-major tile
//   activations      [k/64 chunks][nb rows][128 B], same swizzle (row b,
//                      chunk j at (j ^ (b & 7))); rows >= the batch are zero
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qwen {

constexpr int kTcM = 128;              // output rows per CTA (one M=128 MMA)
constexpr int kTcChunkK = 64;          // k per pipeline stage (one swizzle atom)
constexpr int kTcMaxNb = 256;          // activation rows per launch (MMA N)
constexpr uint32_t kQ4TcChunkBytes = 4608;
constexpr uint32_t kF16TcChunkBytes = kTcM * 128;

inline size_t q4_tc_blob_bytes(int n_rows, int k) {
  return (size_t)(n_rows / kTcM) * (k / kTcChunkK) * kQ4TcChunkBytes;
}
inline size_t f16_tc_blob_bytes(int n_rows, int k) {
  return (size_t)(n_rows / kTcM) * (k / kTcChunkK) * kF16TcChunkBytes;
}
inline size_t act_bytes(int nb, int k) { return (size_t)nb * k * 2; }
// Activation rows padded to the MMA's N granularity.
inline int act_rows(int batch) { return (batch + 15) / 16 * 16; }

struct TcGemmArgs {
  const uint8_t* w = nullptr;  // Q4 or fp16 weight blob
  bool q4 = true;
  const uint8_t* act = nullptr;
  int nb = 16;                 // activation rows of the MMA (multiple of 16, <= 256)
  int act_stride_rows = 0;     // rows per chunk of the activation layout (0: nb)
  int nb_valid = 1;            // rows written out (<= nb)
  int n_rows = 0;              // multiple of 128
  int k = 0;                   // multiple of 64
  int splits = 1;              // K splits (grid.y); must divide k/64
  float* part = nullptr;       // fp32 partials [split][nb_valid][n_rows], or
  __half* out = nullptr;       //   fp16 results out[b * ld_out + n] (splits == 1)
  long long ld_out = 0;
  // SwiGLU epilogue (splits == 1, no part/out): every 128-row tile holds 64
  // gate rows then the 64 matching up rows; row j of the tile pair is written
  // as half(silu(half(g)) * half(u)) into activation tiles of swiglu_nb rows
  // at k index 64 * tile + j (activations.metal:9-27).
  uint8_t* swiglu_act = nullptr;
  int swiglu_nb = 0;
  int* err = nullptr;
  bool pdl = false;            // launch as a programmatic dependent of the previous kernel
  int stages = 0;              // A ring depth, set by launch_tc_gemm
  int xstages = 0;             // activation ring depth, set by launch_tc_gemm
  int raw_stages = 0;          // Q4 raw-weight ring depth, set by launch_tc_gemm
  int unit = 1;                // 64-k chunks per pipeline stage, set by launch_tc_gemm
  int mma_warps = 1;           // issuing warps / accumulators, set by launch_tc_gemm
};

// K splits for a launch: the largest divisor d of the chunk count with
// tiles * d <= sm_count (one wave at one CTA per SM) and at least 2 chunks per
// split (1 if none).
inline int tc_choose_splits(int n_tiles, int n_chunks, int sm_count) {
  int best = 1;
  for (int d = 1; d <= n_chunks; ++d)
    if (n_chunks % d == 0 && n_tiles * d <= sm_count && n_chunks / d >= 2) best = d;
  return best;
}

size_t tc_gemm_smem_bytes(int nb, bool q4, int stages, int xstages, int raw_stages, int unit);
void tc_gemm_rings(int nb, bool q4, int nu, int unit, int* stages, int* xstages, int* raw_stages);
int launch_tc_gemm(const TcGemmArgs& a, cudaStream_t st);

// Weight repacking (device to device) into the blobs above.
int launch_repack_q4_tc(const uint8_t* packed, const __half* scales, int n_rows, int k,
                        uint8_t* blob, cudaStream_t st);
// Rows of a source matrix into half tiles: source row i goes to tile
// i / src_rows_per_tile, tile row dst_row_offset + i % src_rows_per_tile (the
// gate/up pairing: gate with offset 0, up with offset 64, 64 rows per tile).
int launch_repack_q4_tc_rows(const uint8_t* packed, const __half* scales, int n_rows, int k,
                             uint8_t* blob, int src_rows_per_tile, int dst_row_offset,
                             cudaStream_t st);
int launch_repack_f16_tc(const __half* w, int n_rows, int k, uint8_t* blob, cudaStream_t st);
// Row-major fp16 activations x[b * ld + k] (b < rows) -> activation tiles of
// nb rows (rows..nb-1 zero).
int launch_pack_act(const __half* x, long long ld, int rows, int k, int nb, uint8_t* act,
                    cudaStream_t st);
// y[b * ld_y + n] = half(sum_s part[s][b][n] + bias[n]) (bias may be null).
int launch_splits_to_f16(const float* part, int splits, int nb_valid, int n_rows,
                         const __half* bias, __half* y, long long ld_y, cudaStream_t st);

}  // namespace qwen
