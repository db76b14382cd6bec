// fused.h -- layouts and parameters of the fused (persistent) decode step.
//
// Q4 tile layout ("fragment order").  A Q4 matrix [N][K] is cut into 16-row
// tiles; each tile into block pairs (64 k).  One block pair of one tile is
// 576 contiguous bytes:
//   bytes [0, 512):   lane l = 4g + t holds 16 B = the 32-bit words
//                     (row g, block 2p, word t), (row g+8, block 2p, word t),
//                     (row g, block 2p+1, word t), (row g+8, block 2p+1, word t)
//                     of the reference's packed rows (word t of a 16-byte block
//                     = k 8t..8t+7, low nibble first, matmul.metal:37-39)
//   bytes [512, 576): for g = 0..7, four fp16 scales
//                     s(row g, 2p), s(row g+8, 2p), s(row g, 2p+1), s(row g+8, 2p+1)
// "row r" of a tile is a row of the source matrix chosen by the tile's row map
// (RoPE pairs and gate/up pairs share a tile; see layout.cu).  The bytes are a
// pure permutation of the reference's packed bytes and scales.
//
// fp16 LM-head tile layout: 16 vocabulary rows x 1536; per k16 step 512 B,
// lane l = 4g + t holds W[g][16s+4t .. +3] then W[g+8][16s+4t .. +3].
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace qwen {

constexpr int kBpBytes = 576;                   // one block pair of a Q4 tile
constexpr int kBp1536 = 24;                     // block pairs per row, K = 1536
constexpr int kBp8960 = 140;                    // K = 8960
constexpr int kTile1536Bytes = kBp1536 * kBpBytes;   // 13824
constexpr int kTile8960Bytes = kBp8960 * kBpBytes;   // 80640
constexpr int kQKVTiles = 128, kOTiles = 96, kGUTiles = 1120, kDownTiles = 96;
constexpr size_t kLayerQKVOff = 0;
constexpr size_t kLayerOOff = kLayerQKVOff + (size_t)kQKVTiles * kTile1536Bytes;
constexpr size_t kLayerGUOff = kLayerOOff + (size_t)kOTiles * kTile1536Bytes;
constexpr size_t kLayerDownOff = kLayerGUOff + (size_t)kGUTiles * kTile1536Bytes;
constexpr size_t kLayerBlobBytes = kLayerDownOff + (size_t)kDownTiles * kTile8960Bytes;  // 26,320,896

constexpr int kLMTiles = 151936 / 16;           // 9496
constexpr int kLMStepBytes = 512;               // one k16 step of a 16-row fp16 tile
constexpr int kLMTileBytes = 96 * kLMStepBytes; // 49152
constexpr int kLMChunkSteps = 24;               // 12288 B per streamed chunk
constexpr int kDownChunkBp = 24;                // down tiles stream in chunks of 24 block pairs

constexpr int kSlotBytes = kTile1536Bytes;      // ring slot
constexpr int kConsumerWarps = 8;
constexpr int kFusedThreads = (kConsumerWarps + 1) * 32;
constexpr int kAttnWarpsFused = 4;
constexpr int kMaxAttnSplits = 74;
constexpr int kAttnPartWords = 6 * 128 + 12;     // o[6][128], m[6], l[6]

enum FusedPhase : uint16_t { kPhQKV = 0, kPhAttn = 1, kPhO = 2, kPhGU = 3, kPhDown = 4 };
constexpr int kPhasesPerLayer = 5;

// One streamed unit of weights for one CTA.
struct FusedItem {
  uint64_t src;     // byte offset into the Q4 blob or the LM tiles
  uint32_t bytes;
  uint16_t phase;   // layer * 5 + FusedPhase, or n_layers * 5 for the LM head
  uint16_t tile;    // tile index inside its matrix
  uint16_t k0;      // first block pair (Q4) or k16 step (LM) of the chunk
  uint16_t nk;      // block pairs / k16 steps in the chunk
  uint16_t last;    // 1 on the tile's last chunk
  uint16_t seq;     // index of the tile among this CTA's tiles of the phase
};

struct FusedParams {
  const uint8_t* q4;          // Q4 tiles, [layer][kLayerBlobBytes]
  const uint8_t* lm;          // fp16 LM tiles
  const __half* embed;        // [151936][1536] (token gather)
  const __half* norms;        // [layer][2][1536] input / post-attention, then final [1536]
  const __half* qkv_bias;     // [layer][2048] (rows q|k|v, reference order)
  const __half* o_bias;       // [layer][1536]
  const __half* down_bias;    // [layer][1536]
  const float* rope_cs;       // [max_ctx][64][2]
  const FusedItem* items;
  const uint32_t* item_begin; // [grid + 1]
  const uint32_t* seq_ctl;    // SeqCtl of the sequence (read: seq_len, token)
  const uint32_t* epoch;      // step counter (tags of this step's exchanges)
  __half* kc;                 // [layer][max_ctx][256] (reference layout)
  __half* vc;
  uint32_t* x_ll;             // [1536]  tagged fp16 words
  uint32_t* q_ll;             // [1536]
  uint32_t* kv_ll;            // [512]   new k | v of the step
  unsigned long long* attn_part;  // [2][kMaxAttnSplits][kAttnPartWords] tagged fp32 words
  uint32_t* attn_ll;          // [1536]
  uint32_t* h_ll;             // [8960]
  __half* logits;             // [151936]
  int* err;
  int n_layers;
  int max_ctx;
  int kv_layer_stride;        // elements between layers of kc / vc
};

}  // namespace qwen
