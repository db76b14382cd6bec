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
// The down projection (1536 x 8960) is stored block-pair-major instead: unit u
// (block pair u, k = 64u .. 64u+63, u < 140) holds the 96 row tiles' block
// pair u back to back (96 x 576 B), so the CTA that owns unit u -- the 64
// SwiGLU outputs h[64u .. 64u+63], from gate/up tiles 8u .. 8u+7 -- streams
// exactly the down weights those 64 h values multiply.
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
// MLP units: unit u = gate/up tiles 8u .. 8u+7 (h[64u .. 64u+63]) and block
// pair u of every down row tile, streamed as kDownItems items of
// kDownItemTiles row tiles (one ring slot each).
constexpr int kMlpUnits = kBp8960;              // 140
constexpr int kGUTilesPerUnit = kGUTiles / kMlpUnits;  // 8
constexpr int kDownItemTiles = 24;
constexpr int kDownItems = kDownTiles / kDownItemTiles;  // 4
static_assert(kGUTilesPerUnit * kMlpUnits == kGUTiles, "gate/up tiles per MLP unit");
static_assert(kDownItems * kDownItemTiles == kDownTiles, "down items per MLP unit");

constexpr int kLMTiles = 151936 / 16;           // 9496
constexpr int kLMStepBytes = 512;               // one k16 step of a 16-row fp16 tile
constexpr int kLMTileBytes = 96 * kLMStepBytes; // 49152
constexpr int kLMChunkSteps = 24;               // 12288 B per streamed chunk

constexpr int kSlotBytes = kTile1536Bytes;      // ring slot
constexpr int kConsumerWarps = 8;
constexpr int kFusedThreads = kConsumerWarps * 32;
constexpr int kAttnWarpsFused = 4;
constexpr int kMaxAttnSplits = 74;
constexpr int kAttnPartWords = 6 * 128 + 12;     // o[6][128], m[6], l[6]

enum FusedPhase : uint16_t { kPhQKV = 0, kPhAttn = 1, kPhO = 2, kPhGU = 3, kPhDown = 4 };
constexpr int kPhasesPerLayer = 5;
// Trace stamps per CTA: [0] first weight items issued, [1] copies drained at
// exit, [2] consumer start, then per layer kTraceStampsPerLayer stamps (see
// TraceStamp), then LM start, consumer end.  kTsPartialsOut: the CTA's down
// partial sums written; kTsReduced: its rows of the layer output written.
enum TraceStamp : int {
  kTsLayerStart = 0, kTsXReady, kTsQKVDone, kTsAttnDone, kTsOReady, kTsODone, kTsGUReady,
  kTsGUDone, kTsPartialsOut, kTsReduced, kTraceStampsPerLayer
};
// Per CTA: 3 head stamps, 10 per layer, 2 for the LM head, then 7 inside the
// attention unit of the middle layer (start, q/k/v in, warp 0's positions
// done, the unit's warps merged, partials written, partials of all splits in,
// output slice written) on the CTAs that run one.  (Stamps go to shared memory
// during the step; timing the waits of one warp measurably slowed that warp,
// so nothing finer is recorded.)
constexpr int kAttnTraceStamps = 7;
inline int trace_stride_for(int n_layers) {
  return 3 + n_layers * kTraceStampsPerLayer + 2 + kAttnTraceStamps;
}

// One streamed unit of weights for one CTA, packed in 64 bits:
//   bits  0..7   phase  (layer * 5 + FusedPhase, or n_layers * 5 for the LM head)
//   bits  8..21  tile   (tile index inside its matrix; for a down item: the MLP unit)
//   bits 22..29  k0     (first block pair (Q4) or k16 step (LM) of the chunk;
//                        for a down item: its first row tile)
//   bits 30..37  nk     (block pairs / k16 steps / down row tiles in the chunk)
//   bit  38      last   (the tile's last chunk)
//   bits 39..46  seq    (index of the tile among this CTA's tiles of the phase)
// The source offset and byte count follow from these fields (fused.h layouts).
typedef unsigned long long FusedItem;
constexpr int kMaxItemsPerCta = 768;

struct ItemFields {
  int phase, tile, k0, nk, last, seq;
};
__host__ __device__ inline FusedItem pack_item(int phase, int tile, int k0, int nk, int last, int seq) {
  return (FusedItem)phase | ((FusedItem)tile << 8) | ((FusedItem)k0 << 22) |
         ((FusedItem)nk << 30) | ((FusedItem)last << 38) | ((FusedItem)seq << 39);
}
__host__ __device__ inline ItemFields unpack_item(FusedItem w) {
  ItemFields f;
  f.phase = (int)(w & 0xFF);
  f.tile = (int)((w >> 8) & 0x3FFF);
  f.k0 = (int)((w >> 22) & 0xFF);
  f.nk = (int)((w >> 30) & 0xFF);
  f.last = (int)((w >> 38) & 1);
  f.seq = (int)((w >> 39) & 0xFF);
  return f;
}
// Byte offset (into the Q4 blob, or into the LM tiles when phase == lm_phase)
// and byte count of an item.
__host__ __device__ inline void item_source(const ItemFields& f, int lm_phase, size_t* off,
                                            uint32_t* bytes) {
  if (f.phase == lm_phase) {
    *off = (size_t)f.tile * kLMTileBytes + (size_t)f.k0 * kLMStepBytes;
    *bytes = (uint32_t)f.nk * kLMStepBytes;
    return;
  }
  const int layer = f.phase / kPhasesPerLayer, k = f.phase % kPhasesPerLayer;
  size_t base = (size_t)layer * kLayerBlobBytes;
  if (k == kPhQKV) base += kLayerQKVOff;
  else if (k == kPhO) base += kLayerOOff;
  else if (k == kPhGU) base += kLayerGUOff;
  else {
    *off = base + kLayerDownOff + ((size_t)f.tile * kDownTiles + f.k0) * kBpBytes;
    *bytes = (uint32_t)f.nk * kBpBytes;
    return;
  }
  *off = base + (size_t)f.tile * kTile1536Bytes + (size_t)f.k0 * kBpBytes;
  *bytes = (uint32_t)f.nk * kBpBytes;
}

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
  unsigned long long* mlp_part;  // [kMlpUnits][1536] tagged fp32 down partial sums
  __half* logits;             // [151936]
  int* err;
  unsigned long long* trace;  // optional [grid][trace_stride] %globaltimer stamps
  int trace_stride;
  int n_layers;
  int max_ctx;
  int kv_layer_stride;        // elements between layers of kc / vc
  unsigned long long wait_ns; // a dependency wait gives up after this long
  int stall_site;             // test hook: a wait site made to run out (0: none)
};

}  // namespace qwen
