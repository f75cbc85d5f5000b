// Kernel 2: split-KV paged decode attention (sequences with q_len == 1).
//
// Replaces the decode use of candle_flash_attn::flash_attn_varlen_paged_windowed
// at nanovllm_rs/src/layers/attention.rs:43-58 (FA2, SM80 mma.sync atoms).
// Work item = (split, kv head, sequence): one CTA streams one contiguous
// chunk of one sequence's keys for ONE kv head and serves all g = Hq/Hkv
// query heads of that group, so every K/V byte leaves HBM once per group.
//
//  * warp 4 is the TMA producer: it reads the chunk's block-table entries 32
//    pages at a time (one coalesced load), and one lane issues, per 64-token
//    tile, four cp.async.bulk.tensor loads (K and V, two 64-element halves of
//    the 128-wide head each, SWIZZLE_128B) into a 3-stage mbarrier ring;
//  * warps 0-3 each own 16 tokens of every tile: S = Q.K^T and O += P.V run
//    on m16n8k16 MMAs (rows = the g query heads, padded to 16), the online
//    softmax is fp32 with quad shuffles, and P never leaves registers (the S
//    accumulator fragment is re-packed as the A operand of P.V);
//  * warps combine their (m, l, O) through shared memory at the end; a
//    sequence split over several CTAs writes fp32 partials + a base-2 LSE to
//    the workspace and nvkv_decode_combine_kernel merges them.
//
// Roofline: HBM.  Algorithmic bytes per (sequence, kv head) = 2*L*D*2 (K, V)
// plus q/out rows; nothing is re-read across query heads.
//
// The fp8 (e4m3) pool runs the same kernel with kFp8 = true: 128-key tiles
// of codes and row scales, and the transposed e4m3 / f16 products of
// dec8_tile (decode_tile.cuh); see the constants below.
#include <algorithm>

#include "decode_tile.cuh"

namespace nvkv {

constexpr int kDecSmemBytes = kDecStages * kDecStageBytes + 2 * kDecStages * 8 +
                              kDecComputeWarps * 2 * 16 * 4 + 1024;

struct DecodeParams {
  const void* q;
  int64_t q_stride;
  void* out;
  const uint32_t* cu_q;
  const uint32_t* cu_k;
  const uint32_t* block_tables;
  int64_t bt_stride;
  int64_t num_blocks;  // pages (paged) or rows (contiguous)
  int num_q_heads;
  int group;
  int page_size;
  int chunk_tokens;  // keys per split, a multiple of the kernel's tile
  int max_k;         // max_seqlen_k: the block tables cover this many keys
  int64_t num_q_rows;  // rows of q and out
  int max_splits;
  float scale_log2;
  float* ws_o;    // [B][max_splits][Hq][D]
  float* ws_lse;  // [B][max_splits][Hq]
  int* err;
  const float* k_scale;  // fp8 pool: [num_blocks][Hkv][page_size] f32
  const float* v_scale;
  int num_kv_heads;
};

// fp8 (e4m3) pool: 128-key tiles.  The producer stages each tile's K and V
// codes (128 rows x 128 B, one TMA box each, SWIZZLE_128B) and the tile's
// 128 K and 128 V row scales (two 512-byte bulk copies from [page][kv head]
// [row]) in a 3-stage ring, two CTAs per SM; each compute warp runs the
// transposed e4m3 / f16 products of dec8_tile on 32 keys of every tile, on
// the codes in place, so HBM and shared memory each see half the bf16 K/V
// bytes.  A tile carries as
// many bytes as a 64-key bf16 tile: the per-tile costs of the copy pipeline
// (measured to bound 64-key fp8 tiles well below the HBM peak) stay the
// same per byte.
// Measured (8B decode at TP1/2/8, 32B at TP8): 3 stages x 2 CTAs per SM
// beat 2 x 3 everywhere (equal at TP1, 20.6 against 31.2 us at TP8, where
// 256 CTAs fill one wave and each CTA's bytes in flight set its pace).
#ifndef NVKV_DEC8_STAGES
#define NVKV_DEC8_STAGES 3
#endif
#ifndef NVKV_DEC8_CTAS_PER_SM
#define NVKV_DEC8_CTAS_PER_SM 2
#endif
constexpr int kDec8Tile = 128;
constexpr int kDec8Stages = NVKV_DEC8_STAGES;
constexpr int kDec8CtasPerSm = NVKV_DEC8_CTAS_PER_SM;
constexpr int kDec8CodeTile = kDec8Tile * kDecD;   // 16 KB: one K (or V) code tile
constexpr int kDec8ScaleBytes = kDec8Tile * 4;     // one tile's row scales
constexpr int kDec8StageTx = 2 * kDec8CodeTile + 2 * kDec8ScaleBytes;
constexpr int kDec8StageBytes = 34 * 1024;         // keeps every code tile 1024-byte aligned
static_assert(kDec8StageTx <= kDec8StageBytes, "fp8 decode stage layout");
constexpr int kDec8SmemBytes = kDec8Stages * kDec8StageBytes + 2 * kDec8Stages * 8 +
                               kDecComputeWarps * 2 * 16 * 4 + 1024;
static_assert(kDec8Stages * kDec8StageBytes >= kDecComputeWarps * 16 * kDecD * 4,
              "fp8 decode: the final combine reuses the stage memory");
static_assert(kDec8CtasPerSm * (kDec8SmemBytes + 1024) <= 228 * 1024, "fp8 decode: CTAs per SM");
// Groups of 9-16 query heads (two n-tiles of heads: twice the O and Q
// registers) run one CTA per SM, so the tile keeps its registers (255 a
// thread; at 168 it spilled ~1.3 KB), with a 6-stage ring that keeps the
// bytes in flight per SM.  Measured on 64 sequences x 2-4k keys, 16q/1kv:
// 36.0 -> 35.1 us (the bf16 pool: 33.4 us; the shape is latency-bound).
constexpr int kDec8StagesHi = 6;
constexpr int kDec8SmemBytesHi =
    kDec8StagesHi * kDec8StageBytes + 2 * kDec8StagesHi * 8 + kDecComputeWarps * 2 * 16 * 4 + 1024;
static_assert(kDec8SmemBytesHi <= 227 * 1024, "fp8 decode, two head n-tiles: one CTA per SM");

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename T, bool kHi, bool kFp8>
__global__ void __launch_bounds__(kDecThreads, kFp8 ? (kHi ? 1 : kDec8CtasPerSm) : 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const DecodeParams p) {
  constexpr int kStages = kFp8 ? (kHi ? kDec8StagesHi : kDec8Stages) : kDecStages;
  constexpr int kTile = kFp8 ? kDec8Tile : kDecTile;  // keys per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      smem + (kFp8 ? kStages * kDec8StageBytes : kDecStages * kDecStageBytes));
  uint64_t* empty = full + kStages;
  float* red = reinterpret_cast<float*>(empty + kStages);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecComputeWarps);
    }
    fence_mbar_init();
  }
  if (threadIdx.x == kDecComputeWarps * 32) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  // let the (tiny) split-KV combine grid be scheduled while this grid's last
  // wave runs; it waits on griddepcontrol.wait for this grid's results
  pdl_launch_dependents();
  pdl_wait();  // inputs may come from the previous kernel in the stream

  // The producer warp reads its chunk's block-table entries 32 pages at a
  // time, one coalesced load, the first of them together with the sequence
  // lengths (one round trip less before the first TMA), and hands lane 0 each
  // tile's page by a shuffle, so no tile waits on a dependent global load.
  // The first chunk page depends only on the split, and split * chunk_tokens
  // < the plan's key bound <= page_size * bt_stride (validated on the host),
  // so every entry read below lies inside this sequence's table row.
  const int pg_first = (split * p.chunk_tokens) / p.page_size;
  uint32_t ent = 0;
  if (warp == kDecComputeWarps && p.block_tables && pg_first + lane < p.bt_stride)
    ent = __ldg(p.block_tables + (int64_t)b * p.bt_stride + pg_first + lane);

  const uint32_t q0 = p.cu_q[b];
  if (p.cu_q[b + 1] - q0 != 1) return;  // not a decode row: the prefill kernel owns it
  const int k_len = (int)(p.cu_k[b + 1] - p.cu_k[b]);
  const int nsplit = k_len > 0 ? (k_len + p.chunk_tokens - 1) / p.chunk_tokens : 1;
  if (split >= nsplit) return;
  // beyond max_seqlen_k the block table may be shorter; a row past the q/out
  // buffers is neither read nor written
  if (k_len > p.max_k || (int64_t)q0 >= p.num_q_rows) {
    if (threadIdx.x == 0) record_error(p.err, NVKV_DEVERR_SEQLEN);
    return;
  }
  const int tok_begin = split * p.chunk_tokens;
  const int tok_end = min(k_len, tok_begin + p.chunk_tokens);
  const int ntiles = tok_end > tok_begin ? (tok_end - tok_begin + kTile - 1) / kTile : 0;
  if (k_len <= 0 && threadIdx.x == 0) record_error(p.err, NVKV_DEVERR_SEQLEN);
  __syncthreads();

  if (warp == kDecComputeWarps) {
    // ------------------------------ TMA producer ------------------------------
    const int64_t row0 = p.block_tables ? 0 : (int64_t)p.cu_k[b];  // contiguous rows
    int ent_base = 0;  // chunk page held by lane 0's entry
    for (int it = 0; it < ntiles; ++it) {
      const int s = it % kStages;
      const uint32_t ph = (uint32_t)(it / kStages) & 1u;
      const int j0 = tok_begin + it * kTile;
      int64_t row;
      if (p.block_tables) {
        const int pi = j0 / p.page_size - pg_first;  // page within the chunk
        if (pi >= ent_base + 32) {  // warp-uniform: the next 32 entries
          ent_base += 32;
          const int pg = pg_first + ent_base + lane;
          ent = pg < p.bt_stride ? __ldg(p.block_tables + (int64_t)b * p.bt_stride + pg) : 0u;
        }
        uint32_t page = __shfl_sync(0xffffffffu, ent, pi - ent_base);
        if ((int64_t)page >= p.num_blocks) {  // recorded; read as page 0 so the consumers finish
          if (lane == 0) record_error(p.err, NVKV_DEVERR_BLOCK_RANGE);
          page = 0;
        }
        row = (int64_t)page * p.page_size + (j0 % p.page_size);
      } else {
        row = row0 + j0;
      }
      int go = 1;
      if (lane == 0) {
        go = it < kStages || mbar_wait(&empty[s], ph ^ 1u, p.err);
        if (go && kFp8) {
          // scales of the tile's rows: [page][kv head][row in page], 128
          // consecutive floats (tiles never straddle a page)
          uint8_t* st = smem + s * kDec8StageBytes;
          const int64_t si =
              ((row / p.page_size) * p.num_kv_heads + kvh) * p.page_size + row % p.page_size;
          mbar_arrive_expect_tx(&full[s], kDec8StageTx);
          tma_load_3d(st, &tmap_k, &full[s], 0, kvh, (int)row);
          tma_load_3d(st + kDec8CodeTile, &tmap_v, &full[s], 0, kvh, (int)row);
          bulk_load(st + 2 * kDec8CodeTile, p.k_scale + si, kDec8ScaleBytes, &full[s]);
          bulk_load(st + 2 * kDec8CodeTile + kDec8ScaleBytes, p.v_scale + si, kDec8ScaleBytes,
                    &full[s]);
        } else if (go) {
          dec_load_stage(smem + s * kDecStageBytes, &full[s], &tmap_k, &tmap_v, kvh, row);
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
    return;
  }

  // ------------------------------ compute warps ------------------------------
  const int g = p.group;
  const int hq0 = kvh * g;
  const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)q0 * p.q_stride + (int64_t)hq0 * kDecD;
  float* ofin = reinterpret_cast<float*>(smem);  // [warp][16][128] fp32 = 32 KB, after the loop
  if constexpr (kFp8) {
    constexpr int kP = Dec8Q<T>::kPieces, kNt = kHi ? 2 : 1;
    uint32_t qb[kP][kNt][8];
    const float s_log2 = p.scale_log2 * dec8_load_q<T, kP, kNt>(qb, qrow, g, lane);
    Dec8State<kNt> st;
    st.reset();
    const int wtok = warp * 32;  // this warp's keys of every tile
    for (int it = 0; it < ntiles; ++it) {
      const int s = it % kStages;
      const uint32_t ph = (uint32_t)(it / kStages) & 1u;
      if (!mbar_wait(&full[s], ph, p.err)) break;
      uint8_t* stage = smem + s * kDec8StageBytes;
      const uint32_t kbase = smem_u32(stage);
      const float* sc = reinterpret_cast<const float*>(stage + 2 * kDec8CodeTile);
      const int valid = tok_end - (tok_begin + it * kDec8Tile + wtok);  // this warp's keys
      if (valid >= 32)
        dec8_tile<kP, kNt, false>(qb, st, kbase, kbase + kDec8CodeTile, sc, sc + kDec8Tile, wtok,
                                  valid, s_log2, lane);
      else if (valid > 0)
        dec8_tile<kP, kNt, true>(qb, st, kbase, kbase + kDec8CodeTile, sc, sc + kDec8Tile, wtok,
                                 valid, s_log2, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    dec8_put_ml<kNt>(st, red, warp, lane);
    named_bar_sync(1, kDecComputeWarps * 32);  // all loops done: stage memory is free
    dec8_put_o<kNt>(st, red, ofin + warp * 16 * kDecD, kDecComputeWarps, lane);
  } else {
    const int r0 = lane >> 2, r1 = r0 + 8;
    const int cq = (lane & 3) * 2;
    uint32_t qa[8][4];
    dec_load_q<T>(qa, qrow, g, lane);
    DecState st;
    st.reset();
    for (int it = 0; it < ntiles; ++it) {
      const int s = it % kStages;
      const uint32_t ph = (uint32_t)(it / kStages) & 1u;
      if (!mbar_wait(&full[s], ph, p.err)) break;
      const uint32_t kbase = smem_u32(smem + s * kDecStageBytes);
      const int valid = tok_end - (tok_begin + it * kDecTile + warp * 16);  // keys of this slice
      if (valid > 0)
        dec_tile<T, kHi>(qa, st, kbase, kbase + kDecTileBytes, warp * 16, valid, p.scale_log2,
                         lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ------------------------------ warp combine ------------------------------
    float l0 = st.l0, l1 = st.l1;
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if ((lane & 3) == 0) {
      red[(warp * 2 + 0) * 16 + r0] = st.m0;
      red[(warp * 2 + 1) * 16 + r0] = l0;
      red[(warp * 2 + 0) * 16 + r1] = st.m1;
      red[(warp * 2 + 1) * 16 + r1] = l1;
    }
    named_bar_sync(1, kDecComputeWarps * 32);  // all loops done: stage memory is free

    float ms0 = -INFINITY, ms1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecComputeWarps; ++w) {
      ms0 = fmaxf(ms0, red[(w * 2) * 16 + r0]);
      ms1 = fmaxf(ms1, red[(w * 2) * 16 + r1]);
    }
    const float f0 = exp2f(st.m0 - (ms0 == -INFINITY ? 0.f : ms0));
    const float f1 = exp2f(st.m1 - (ms1 == -INFINITY ? 0.f : ms1));
    float* ow = ofin + warp * 16 * kDecD;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int d = n * 8 + cq;
      *reinterpret_cast<float2*>(ow + r0 * kDecD + d) = make_float2(st.o[n][0] * f0, st.o[n][1] * f0);
      *reinterpret_cast<float2*>(ow + r1 * kDecD + d) = make_float2(st.o[n][2] * f1, st.o[n][3] * f1);
    }
  }
  named_bar_sync(1, kDecComputeWarps * 32);

  const int tid = threadIdx.x;  // 0..127 == d
  for (int r = 0; r < g; ++r) {
    float ms = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecComputeWarps; ++w) ms = fmaxf(ms, red[(w * 2) * 16 + r]);
    const float mu = ms == -INFINITY ? 0.f : ms;
    float ls = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecComputeWarps; ++w) {
      ls += red[(w * 2 + 1) * 16 + r] * exp2f(red[(w * 2) * 16 + r] - mu);
      acc += ofin[(w * 16 + r) * kDecD + (kFp8 ? dec8_ofin_col(tid, r) : tid)];
    }
    const float val = ls > 0.f ? acc / ls : 0.f;
    const int hq = hq0 + r;
    if (nsplit == 1) {
      T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)q0 * p.num_q_heads + hq) * kDecD;
      dst[tid] = DT<T>::from_f(val);
    } else {
      const int64_t wi = ((int64_t)b * p.max_splits + split) * p.num_q_heads + hq;
      p.ws_o[wi * kDecD + tid] = val;
      if (tid == 0) p.ws_lse[wi] = ls > 0.f ? ms + log2f(ls) : -INFINITY;
    }
  }
}

// Merge of the split-KV partials of one (sequence, query head): weights
// 2^(lse_s - max lse), the standard log-sum-exp combine.
// Launched as a programmatic dependent of the decode kernel: its CTAs may be
// scheduled while the decode grid drains, and griddepcontrol.wait holds them
// until that grid has completed and its partials are visible.
template <typename T>
__global__ void __launch_bounds__(kDecD) decode_combine_kernel(const DecodeParams p) {
  pdl_wait();
  const int hq = blockIdx.x, b = blockIdx.y;
  const uint32_t q0 = p.cu_q[b];
  if (p.cu_q[b + 1] - q0 != 1) return;
  const int k_len = (int)(p.cu_k[b + 1] - p.cu_k[b]);
  const int nsplit = k_len > 0 ? (k_len + p.chunk_tokens - 1) / p.chunk_tokens : 1;
  // the decode grid wrote no partials for these (and reported them)
  if (nsplit <= 1 || k_len > p.max_k || (int64_t)q0 >= p.num_q_rows) return;
  const int64_t base = (int64_t)b * p.max_splits * p.num_q_heads + hq;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, p.ws_lse[base + (int64_t)s * p.num_q_heads]);
  const float mu = mx == -INFINITY ? 0.f : mx;
  float wsum = 0.f, acc = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const int64_t wi = base + (int64_t)s * p.num_q_heads;
    const float w = exp2f(p.ws_lse[wi] - mu);
    wsum += w;
    acc += w * p.ws_o[wi * kDecD + threadIdx.x];
  }
  T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)q0 * p.num_q_heads + hq) * kDecD;
  dst[threadIdx.x] = DT<T>::from_f(wsum > 0.f ? acc / wsum : 0.f);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Split-KV plan: enough CTAs for ~3 resident waves (a wave = 148 SMs x the
// kernel's CTAs per SM: 2 for bf16/f16 pools, kDec8CtasPerSm for fp8), but
// never chunks shorter than 12 tiles (768 keys): a sweep over the decode
// shapes of configs 2, 4 (TP1, TP8) and 5 found this the best or equal-best
// everywhere (shorter chunks pay per-CTA setup and merge work on small
// per-GPU batches).  Exception: when one CTA per (sequence, kv head) already
// fills >= 80 % of a resident wave and no sequence exceeds
// NVKV_DECODE_ONE_WAVE_MAX_TILES tiles, nothing is split -- a single wave
// with no combine beats 1.7 waves plus a combine (8B TP8, 256 seqs: 37.2 ->
// 31.1 us at ctx <= 1536, 54.7 -> 45.6 us at ctx <= 2560).  The cost is
// bounded by the tile cap: one long sequence among short ones then runs
// unsplit (+1.3 us measured at 24 tiles).
#ifndef NVKV_DECODE_WAVES
#define NVKV_DECODE_WAVES 3
#endif
#ifndef NVKV_DECODE_MIN_TILES
#define NVKV_DECODE_MIN_TILES 12
#endif
#ifndef NVKV_DECODE_ONE_WAVE_MAX_TILES
#define NVKV_DECODE_ONE_WAVE_MAX_TILES 48
#endif
void decode_plan(int num_seqs, int num_kv_heads, int max_seqlen_k, bool fp8, int* chunk_tokens,
                 int* max_splits) {
  const int ctas_per_sm = fp8 ? kDec8CtasPerSm : 2;
  const int tile = fp8 ? kDec8Tile : kDecTile;
  const int tiles = max_seqlen_k > 0 ? (max_seqlen_k + tile - 1) / tile : 1;
  const int64_t items = (int64_t)num_seqs * num_kv_heads;
  const int64_t wave = 148 * (int64_t)ctas_per_sm;
  const int64_t target = NVKV_DECODE_WAVES * wave;
  int splits = (int)((target + items - 1) / items);
  // the limits are stated in 64-key units
  const int min_tiles = std::max(1, NVKV_DECODE_MIN_TILES * kDecTile / tile);
  const int max_by_len = (tiles + min_tiles - 1) / min_tiles;
  if (splits > max_by_len) splits = max_by_len;
  if (items * 5 >= wave * 4 && tiles * tile <= NVKV_DECODE_ONE_WAVE_MAX_TILES * kDecTile)
    splits = 1;
  if (splits < 1) splits = 1;
  const int tiles_per_split = (tiles + splits - 1) / splits;
  *chunk_tokens = tiles_per_split * tile;
  *max_splits = (tiles + tiles_per_split - 1) / tiles_per_split;
}

size_t decode_workspace_bytes(int num_seqs, int num_q_heads, int num_kv_heads, int max_seqlen_k,
                              bool fp8) {
  int chunk, splits;
  decode_plan(num_seqs, num_kv_heads, max_seqlen_k, fp8, &chunk, &splits);
  if (splits <= 1) return 0;
  const size_t n = (size_t)num_seqs * splits * num_q_heads;
  return n * kDecD * sizeof(float) + n * sizeof(float) + 256;
}

// The combine launch overlaps the decode grid's tail (programmatic stream
// serialisation); the kernel's griddepcontrol.wait keeps the data order.
static int launch_combine(void (*kern)(DecodeParams), const DecodeParams& p, const AttnArgs& a) {
  return launch_pdl(kern, dim3(a.hq, a.num_seqs), dim3(kDecD), 0, a.stream, "decode combine launch",
                    p);
}

template <typename T, bool kFp8>
static int launch_decode_grid(bool hi, dim3 grid, const CUtensorMap& mk, const CUtensorMap& mv,
                              const DecodeParams& p, cudaStream_t stream) {
  auto kern = hi ? paged_decode_kernel<T, true, kFp8> : paged_decode_kernel<T, false, kFp8>;
  const int smem = kFp8 ? (hi ? kDec8SmemBytesHi : kDec8SmemBytes) : kDecSmemBytes;
  constexpr int threads = kDecThreads;
  static unsigned long long attr_done[2] = {0, 0};  // per instantiation and kHi
  int rc = ensure_smem_attr((const void*)kern, smem, &attr_done[hi]);
  if (!rc)
    rc = launch_pdl(kern, grid, dim3(threads), smem, stream, "paged decode launch", mk, mv, p);
  return rc;
}

int launch_paged_decode(const AttnArgs& a) {
  const bool fp8 = a.k_scale != nullptr;
  int chunk, splits;
  decode_plan(a.num_seqs, a.hkv, a.max_k, fp8, &chunk, &splits);
  const int64_t rows = a.block_tables ? a.num_blocks * a.page : a.num_blocks;
  CUtensorMap mk, mv;
  int rc;
  if (fp8) {  // paged only; rows of Hkv x 128 one-byte codes
    rc = encode_kv_tensor_map_u8(&mk, a.k_cache, kDecD, a.hkv, rows, a.kv_stride, kDec8Tile);
    if (!rc)
      rc = encode_kv_tensor_map_u8(&mv, a.v_cache, kDecD, a.hkv, rows, a.kv_stride, kDec8Tile);
  } else {
    rc = encode_kv_tensor_map(&mk, a.k_cache, kDecD, a.hkv, rows, a.kv_stride * 2, 64, kDecTile,
                              true);
    if (!rc)
      rc = encode_kv_tensor_map(&mv, a.v_cache, kDecD, a.hkv, rows, a.kv_stride * 2, 64,
                                kDecTile, true);
  }
  if (rc) return rc;
  DecodeParams p;
  p.q = a.q;
  p.q_stride = a.q_stride;
  p.out = a.out;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.num_blocks = a.num_blocks;
  p.num_q_heads = a.hq;
  p.group = a.hq / a.hkv;
  p.page_size = a.page;
  p.chunk_tokens = chunk;
  p.max_k = a.max_k;
  p.num_q_rows = a.num_q_rows;
  p.max_splits = splits;
  p.scale_log2 = a.scale * kLog2e;
  p.ws_o = nullptr;
  p.ws_lse = nullptr;
  p.err = device_error_word();
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.num_kv_heads = a.hkv;
  if (splits > 1) {
    const size_t n = (size_t)a.num_seqs * splits * a.hq;
    p.ws_o = reinterpret_cast<float*>(a.ws);
    p.ws_lse = p.ws_o + n * kDecD;
  }
  dim3 grid(splits, a.hkv, a.num_seqs);
  // group sizes up to 8 leave fragment rows 8..15 as padding (kHi = false)
  const bool hi = p.group > 8;
  if (a.dtype == NVKV_DTYPE_BF16) {
    rc = fp8 ? launch_decode_grid<__nv_bfloat16, true>(hi, grid, mk, mv, p, a.stream)
             : launch_decode_grid<__nv_bfloat16, false>(hi, grid, mk, mv, p, a.stream);
    if (!rc && splits > 1) rc = launch_combine(decode_combine_kernel<__nv_bfloat16>, p, a);
  } else {
    rc = fp8 ? launch_decode_grid<__half, true>(hi, grid, mk, mv, p, a.stream)
             : launch_decode_grid<__half, false>(hi, grid, mk, mv, p, a.stream);
    if (!rc && splits > 1) rc = launch_combine(decode_combine_kernel<__half>, p, a);
  }
  return rc;
}

}  // namespace nvkv
