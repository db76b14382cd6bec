// layout.cu -- builds the fused decode step's weight layouts on the device
// (Q4 fragment-order tiles, fp16 LM-head tiles), the RoPE cos/sin table and
// the per-CTA work schedule.  See fused.h for the byte layouts.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "engine.h"
#include "fused.h"
#include "qwen_common.cuh"
#include "status.h"

namespace qwen {

enum RowMap : int { kMapPlain = 0, kMapRopePairs = 1, kMapGateUp = 2 };

// Up to three reference-layout matrices with the same K, concatenated by rows.
struct Q4Sources {
  const uint8_t* packed[3];
  const __half* scales[3];
  int rows[3];
};

// Row (in the concatenated row space) of row r (0..15) of tile `tile`.
//   RopePairs: tile = head*8 + j holds dims 8j..8j+7 (r < 8) and
//              64+8j..64+8j+7 (r >= 8) of head `head`, so the lane that owns
//              rows g and g+8 owns a rotate-half pair (rope.metal:21-22).
//   GateUp:    tile t holds gate rows 8t..8t+7 and up rows 8t..8t+7
//              (activations.metal:9-27 combines them element-wise).
__device__ __forceinline__ int tile_row(int map, int tile, int r) {
  if (map == kMapRopePairs) {
    const int head = tile >> 3, j = tile & 7;
    return head * 128 + (r < 8 ? 8 * j + r : 64 + 8 * j + (r - 8));
  }
  if (map == kMapGateUp) return r < 8 ? 8 * tile + r : kInter + 8 * tile + (r - 8);
  return 16 * tile + r;
}

__device__ __forceinline__ void locate(const Q4Sources& s, int row, int& m, int& local) {
  m = 0;
  local = row;
  while (m < 2 && local >= s.rows[m]) {
    local -= s.rows[m];
    ++m;
  }
}

// bp_major: block pair p of tile `tile` goes to (p * n_tiles + tile) instead of
// (tile * P + p) -- the MLP-unit order of the down projection (fused.h).
__global__ void k_repack_q4(Q4Sources src, int k, int n_tiles, int map, int bp_major,
                            uint8_t* __restrict__ dst) {
  const int P = k / 64;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_tiles * P * 32) return;
  const int lane = (int)(idx & 31);
  const long long tp = idx >> 5;
  const int p = (int)(tp % P), tile = (int)(tp / P);
  const int g = lane >> 2, t = lane & 3;
  int mg, lg, mg8, lg8;
  locate(src, tile_row(map, tile, g), mg, lg);
  locate(src, tile_row(map, tile, g + 8), mg8, lg8);
  const size_t rb = (size_t)k / 2;
  const uint8_t* rowg = src.packed[mg] + (size_t)lg * rb + 4 * t;
  const uint8_t* rowg8 = src.packed[mg8] + (size_t)lg8 * rb + 4 * t;
  uint4 w;
  w.x = *reinterpret_cast<const uint32_t*>(rowg + 16 * (2 * p));
  w.y = *reinterpret_cast<const uint32_t*>(rowg8 + 16 * (2 * p));
  w.z = *reinterpret_cast<const uint32_t*>(rowg + 16 * (2 * p + 1));
  w.w = *reinterpret_cast<const uint32_t*>(rowg8 + 16 * (2 * p + 1));
  uint8_t* out = dst + (bp_major ? (size_t)p * n_tiles + tile : (size_t)tile * P + p) * kBpBytes;
  reinterpret_cast<uint4*>(out)[lane] = w;
  if (t == 0) {
    const int nb = k / 32;
    const __half* sg = src.scales[mg] + (size_t)lg * nb;
    const __half* sg8 = src.scales[mg8] + (size_t)lg8 * nb;
    __half s4[4] = {sg[2 * p], sg8[2 * p], sg[2 * p + 1], sg8[2 * p + 1]};
    *reinterpret_cast<uint2*>(out + 512 + 8 * g) = *reinterpret_cast<uint2*>(s4);
  }
}

__global__ void k_repack_lm(const __half* __restrict__ w, uint8_t* __restrict__ dst) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)kLMTiles * 96 * 32;
  if (idx >= total) return;
  const int lane = (int)(idx & 31);
  const long long ts = idx >> 5;
  const int s = (int)(ts % 96), tile = (int)(ts / 96);
  const int g = lane >> 2, t = lane & 3;
  const uint2 a = *reinterpret_cast<const uint2*>(w + (size_t)(16 * tile + g) * kHidden + 16 * s + 4 * t);
  const uint2 b = *reinterpret_cast<const uint2*>(w + (size_t)(16 * tile + g + 8) * kHidden + 16 * s + 4 * t);
  reinterpret_cast<uint4*>(dst + ((size_t)tile * 96 + s) * kLMStepBytes)[lane] = make_uint4(a.x, a.y, b.x, b.y);
}

static int repack(const Q4Sources& s, int k, int n_tiles, int map, uint8_t* dst, cudaStream_t st,
                  int bp_major = 0) {
  const long long n = (long long)n_tiles * (k / 64) * 32;
  k_repack_q4<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(s, k, n_tiles, map, bp_major, dst);
  return launch_status("repack_q4");
}

// ------------------------------------------------------------ schedule ----
// Assignment of every streamed tile of a step to CTAs.  Phase order per
// layer: QKV, (attention: no weights), O, gate/up, down; then the LM head.
//   QKV: the first 128 CTAs, one tile each (the attention units use the last
//        CTAs);
//   O:   one tile per CTA, on the CTAs with the least bytes so far;
//   MLP: unit u (gate/up tiles 8u .. 8u+7, then its down strip as kDownItems
//        items) on CTA u, so every CTA below kMlpUnits owns one unit (the
//        grid must have at least kMlpUnits CTAs);
//   LM head: tile t on CTA t % grid, in chunks of kLMChunkSteps.
// Returns false when the grid is too small for the MLP units.
static bool build_schedule(int n_layers, int grid, std::vector<FusedItem>& items,
                           std::vector<uint32_t>& begin) {
  items.clear();
  begin.assign(grid + 1, 0);
  if (grid < kMlpUnits) return false;
  std::vector<std::vector<FusedItem>> per(grid);
  std::vector<double> load(grid, 0.0);
  std::vector<std::vector<int>> tiles_in_phase(grid, std::vector<int>(n_layers * kPhasesPerLayer + 1, 0));
  auto add_tile = [&](int cta, uint16_t phase, int tile, int n_k, int chunk_k, int unit_bytes) {
    const int seq = tiles_in_phase[cta][phase]++;
    for (int k0 = 0; k0 < n_k; k0 += chunk_k) {
      const int nk = std::min(chunk_k, n_k - k0);
      per[cta].push_back(pack_item(phase, tile, k0, nk, k0 + nk >= n_k, seq));
      load[cta] += (double)nk * unit_bytes;
    }
  };
  for (int l = 0; l < n_layers; ++l) {
    const uint16_t ph = (uint16_t)(l * kPhasesPerLayer);
    for (int t = 0; t < kQKVTiles; ++t) add_tile(t % grid, ph + kPhQKV, t, kBp1536, kBp1536, kBpBytes);
    for (int t = 0; t < kOTiles; ++t) {
      int best = -1;
      for (int c = 0; c < grid; ++c)
        if (tiles_in_phase[c][ph + kPhO] == 0 && (best < 0 || load[c] < load[best])) best = c;
      add_tile(best, ph + kPhO, t, kBp1536, kBp1536, kBpBytes);
    }
    for (int u = 0; u < kMlpUnits; ++u) {
      for (int j = 0; j < kGUTilesPerUnit; ++j)
        add_tile(u, ph + kPhGU, kGUTilesPerUnit * u + j, kBp1536, kBp1536, kBpBytes);
      // the unit's down strip: kDownTiles row tiles of one block pair each
      add_tile(u, ph + kPhDown, u, kDownTiles, kDownItemTiles, kBpBytes);
    }
  }
  const uint16_t lm_phase = (uint16_t)(n_layers * kPhasesPerLayer);
  // The LM head is its own phase after the last layer (a ring slot holds one
  // chunk, so it cannot be fetched much earlier): balance its tiles alone,
  // not the bytes of the whole step.
  for (int t = 0; t < kLMTiles; ++t) add_tile(t % grid, lm_phase, t, 96, kLMChunkSteps, kLMStepBytes);
  for (int c = 0; c < grid; ++c) {
    if (per[c].size() > (size_t)kMaxItemsPerCta) per[c].clear();  // reported by the caller
    begin[c] = (uint32_t)items.size();
    items.insert(items.end(), per[c].begin(), per[c].end());
  }
  begin[grid] = (uint32_t)items.size();
  return true;
}

// RoPE cos/sin per position: theta = pos * 1e6^(-2i/128) in fp32 with libm,
// exactly as rope.metal:25-32 evaluates it.  Table [ctx][64][2] (cos, sin).
int upload_rope_table(float** cs_dev, int* ctx, int max_ctx, cudaStream_t st) {
  if (*ctx < max_ctx) {
    if (*cs_dev) cudaFree(*cs_dev);
    *cs_dev = nullptr;
    *ctx = 0;
    QWEN_CUDA(cudaMalloc((void**)cs_dev, (size_t)max_ctx * 128 * sizeof(float)), "cudaMalloc(rope)");
    *ctx = max_ctx;
  }
  float inv[64];
  rope_inv_freq(inv);
  std::vector<float> cs((size_t)max_ctx * 128);
  for (int pos = 0; pos < max_ctx; ++pos)
    for (int i = 0; i < 64; ++i) {
      const float theta = (float)pos * inv[i];
      cs[(size_t)pos * 128 + 2 * i] = std::cos(theta);
      cs[(size_t)pos * 128 + 2 * i + 1] = std::sin(theta);
    }
  QWEN_CUDA(cudaMemcpyAsync(*cs_dev, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice, st),
            "memcpy rope");
  QWEN_CUDA(cudaStreamSynchronize(st), "sync");
  return QWEN_OK;
}

int build_fused_weights(QwenModel& m, int max_ctx, cudaStream_t st) {
  FusedWeights& f = m.fused;
  auto alloc = [&](void** p, size_t bytes) { return cuda_status(cudaMalloc(p, bytes), "cudaMalloc(fused)"); };
  if (!f.blob) {
    f.blob_bytes = (size_t)m.n_layers * kLayerBlobBytes;
    QWEN_TRY(alloc((void**)&f.blob, f.blob_bytes));
    QWEN_TRY(alloc((void**)&f.lm_tiles, (size_t)kLMTiles * kLMTileBytes));
    QWEN_TRY(alloc((void**)&f.norms, ((size_t)m.n_layers * 2 + 1) * kHidden * 2));
    QWEN_TRY(alloc((void**)&f.qkv_bias, (size_t)m.n_layers * kQKVRows * 2));
    QWEN_TRY(alloc((void**)&f.o_bias, (size_t)m.n_layers * kHidden * 2));
    QWEN_TRY(alloc((void**)&f.down_bias, (size_t)m.n_layers * kHidden * 2));
  }
  for (int l = 0; l < m.n_layers; ++l) {
    const QwenLayer& L = m.layers[l];
    uint8_t* lb = f.blob + (size_t)l * kLayerBlobBytes;
    Q4Sources qkv{{L.q.packed, L.k.packed, L.v.packed}, {L.q.scales, L.k.scales, L.v.scales},
                  {kHidden, kKVDim, kKVDim}};
    QWEN_TRY(repack(qkv, kHidden, kQKVTiles, kMapRopePairs, lb + kLayerQKVOff, st));
    Q4Sources o{{L.o.packed, nullptr, nullptr}, {L.o.scales, nullptr, nullptr}, {kHidden, 0, 0}};
    QWEN_TRY(repack(o, kHidden, kOTiles, kMapPlain, lb + kLayerOOff, st));
    Q4Sources gu{{L.gate.packed, L.up.packed, nullptr}, {L.gate.scales, L.up.scales, nullptr},
                 {kInter, kInter, 0}};
    QWEN_TRY(repack(gu, kHidden, kGUTiles, kMapGateUp, lb + kLayerGUOff, st));
    Q4Sources dn{{L.down.packed, nullptr, nullptr}, {L.down.scales, nullptr, nullptr}, {kHidden, 0, 0}};
    QWEN_TRY(repack(dn, kInter, kDownTiles, kMapPlain, lb + kLayerDownOff, st, 1));
    QWEN_CUDA(cudaMemcpyAsync(f.norms + (size_t)(2 * l) * kHidden, L.input_norm, kHidden * 2,
                              cudaMemcpyDeviceToDevice, st), "memcpy");
    QWEN_CUDA(cudaMemcpyAsync(f.norms + (size_t)(2 * l + 1) * kHidden, L.post_attn_norm, kHidden * 2,
                              cudaMemcpyDeviceToDevice, st), "memcpy");
    QWEN_CUDA(cudaMemcpyAsync(f.qkv_bias + (size_t)l * kQKVRows, L.qkv_bias, kQKVRows * 2,
                              cudaMemcpyDeviceToDevice, st), "memcpy");
    QWEN_CUDA(cudaMemcpyAsync(f.o_bias + (size_t)l * kHidden, L.o_bias, kHidden * 2,
                              cudaMemcpyDeviceToDevice, st), "memcpy");
    QWEN_CUDA(cudaMemcpyAsync(f.down_bias + (size_t)l * kHidden, L.down_bias, kHidden * 2,
                              cudaMemcpyDeviceToDevice, st), "memcpy");
  }
  QWEN_CUDA(cudaMemcpyAsync(f.norms + (size_t)(2 * m.n_layers) * kHidden, m.final_norm, kHidden * 2,
                            cudaMemcpyDeviceToDevice, st), "memcpy");
  {
    const long long n = (long long)kLMTiles * 96 * 32;
    k_repack_lm<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(m.embed, f.lm_tiles);
    QWEN_TRY(launch_status("repack_lm"));
  }
  QWEN_TRY(upload_rope_table(&f.rope_cs, &f.rope_ctx, max_ctx, st));
  // Work schedule for the current device's SM count.
  int dev = 0, sms = 0;
  QWEN_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  QWEN_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "attr");
  std::vector<FusedItem> items;
  std::vector<uint32_t> begin;
  if (!build_schedule(m.n_layers, sms, items, begin))
    return set_error(QWEN_ERR_STATE, "the fused step needs at least %d SMs (device has %d)", kMlpUnits,
                     sms);
  for (int c = 0; c < sms; ++c)
    if (begin[c + 1] == begin[c])
      return set_error(QWEN_ERR_STATE, "fused schedule: CTA %d has no work or more than %d items", c,
                       kMaxItemsPerCta);
  if (f.items) cudaFree(f.items);
  if (f.item_begin) cudaFree(f.item_begin);
  f.items = nullptr;
  f.item_begin = nullptr;
  QWEN_TRY(alloc((void**)&f.items, items.size() * sizeof(FusedItem)));
  QWEN_TRY(alloc((void**)&f.item_begin, begin.size() * sizeof(uint32_t)));
  QWEN_CUDA(cudaMemcpy(f.items, items.data(), items.size() * sizeof(FusedItem), cudaMemcpyHostToDevice), "memcpy");
  QWEN_CUDA(cudaMemcpy(f.item_begin, begin.data(), begin.size() * sizeof(uint32_t), cudaMemcpyHostToDevice), "memcpy");
  f.grid = sms;
  QWEN_CUDA(cudaStreamSynchronize(st), "sync");
  return QWEN_OK;
}

}  // namespace qwen

// Test hook (not part of the public header): the fused step's work schedule
// for n_layers layers on `grid` CTAs, exactly as build_fused_weights builds it.
// Writes the packed items (fused.h: FusedItem) into items_out (capacity
// items_cap) and the per-CTA begin offsets into begin_out[grid + 1].  Host
// arithmetic only.  Returns the item count, or -1 when an argument is out of
// range or the capacity is too small.
extern "C" long long qwen_fused_schedule(int n_layers, int grid, unsigned long long* items_out,
                                         long long items_cap, unsigned int* begin_out) {
  if (n_layers < 1 || n_layers > 64 || grid < 1 || grid > 1024 || !items_out || !begin_out) return -1;
  std::vector<qwen::FusedItem> items;
  std::vector<uint32_t> begin;
  if (!qwen::build_schedule(n_layers, grid, items, begin)) return -1;
  if ((long long)items.size() > items_cap) return -1;
  std::copy(items.begin(), items.end(), items_out);
  std::copy(begin.begin(), begin.end(), begin_out);
  return (long long)items.size();
}
