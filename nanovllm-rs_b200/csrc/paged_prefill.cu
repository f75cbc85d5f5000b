// Kernel 3: varlen (paged) causal prefill attention on tcgen05 tensor cores.
//
// Replaces the prefill / mixed-batch uses of candle_flash_attn
// (flash_attn_varlen and flash_attn_varlen_paged_windowed, nanovllm_rs/src/
// layers/attention.rs:43-73; FA2 with SM80 mma.sync) for every sequence
// whose q_len > 1 (q_len == 1 rows run on the decode kernel).
//
// One work item = 128 query rows x TWO query heads of the same kv group
// (slots A and B; one slot when the group size is odd).  Both slots read the
// same K/V tiles, so every K/V tile is fetched once per head pair, and the
// two softmax warpgroups ping-pong against the tensor core.  The kernel is
// persistent (one CTA per SM walking its work items, see pf_work).  10 warps:
//   warp 0      TMA producer: Q_A/Q_B per item, then K_j, V_j (128 keys each,
//               pages resolved through block_tables) through a 5-slot ring,
//               SWIZZLE_128B, each CTA loading its own tiles;
//   warp 1      allocates all 512 TMEM columns (S_A, S_B, O_A, O_B) and
//               issues every tcgen05.mma.cta_group::1.kind::f16 from one
//               thread in the order  PV_A(j), S_A(j+1), PV_B(j), S_B(j+1),
//               so the tensor core computes one slot while the other slot's
//               softmax runs; tcgen05.commit arrives on the mbarriers;
//   warps 2-5   softmax warpgroup of slot A, warps 6-9 of slot B: thread r
//               owns query row r (TMEM lane r).  Per key tile it loads its
//               whole S row from TMEM (four tcgen05.ld 32x32b.x32, one wait),
//               masks (causal, bottom-right: key j visible to query i iff
//               j <= i + k_len - q_len), takes the exact row max from
//               registers, and rescales the TMEM O row (tcgen05.ld/st) only
//               when the max grew by more than 2^8 -- otherwise it keeps the
//               stale max, whose exponentials stay <= 256 and exact enough in
//               fp32/bf16 -- then writes P = 2^(s*scale - m) as 16-bit pairs
//               back into the first 64 columns of its S region (tcgen05.st).
//               The P.V MMA takes P from TMEM as its A operand, so no shared
//               memory holds P and the 64 KB it would take deepen the K/V
//               ring; S_x(j+1) may overwrite P_x(j) because it is issued
//               after PV_x(j) on the in-order tensor pipe.  Seven exponential
//               pairs in eight run on the MUFU ex2 unit, one on a polynomial
//               on the FMA pipe (kPfPolyEvery); the scaling FMAs and the row
//               sum use packed f32x2 instructions.
//   O accumulates in TMEM across key tiles (PV MMAs chain with
//   accumulate = 1); the epilogue divides by the row sum and stores bf16/f16.
// Roofline: tensor cores; flops = 4 * D * (visible (query, key) pairs).
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace nvkv {

constexpr int kPfD = 128;
constexpr int kPfBM = 128;
constexpr int kPfBN = 128;
constexpr int kPfSlots = 5;                 // K/V ring: K_j and V_j each take one slot
constexpr int kPfThreads = 10 * 32;
constexpr int kPfHalf = 128 * 128;          // 128 rows x 128 B (64 elements)
constexpr int kPfTile = 2 * kPfHalf;        // 32 KB: 128 rows x 128 elements
constexpr int kPfOffQA = 0;
constexpr int kPfOffQB = kPfOffQA + kPfTile;
constexpr int kPfOffKV = kPfOffQB + kPfTile;
constexpr int kPfOffBar = kPfOffKV + kPfSlots * kPfTile;
constexpr int kPfNumBars = 2 + 2 * kPfSlots + 6;
constexpr int kPfSmemBytes = kPfOffBar + kPfNumBars * 8 + 16 + 1024;
constexpr uint32_t kPfTmemCols = 512;
constexpr int kPfCtas = 148;  // B200 SMs
// Direct enumeration of every candidate (q tile, head slot, sequence) is kept
// when nearly all candidates are real work (the query tokens fill at least
// kPfDirectFill of the candidate q tiles: uniform prompts) or the batch is
// tiny (at most kPfDirectItemsPerCta candidates per CTA); otherwise the work
// plan goes first.  Measured: 16 x 1024 prompts, direct 196.5 us / plan
// 211.6 us; 8 prompts U[128, 2048], direct 181.9 / plan 156.5; 120 decodes +
// those 8 prompts, direct 362 / plan 267.
constexpr int kPfDirectItemsPerCta = 2;
constexpr double kPfDirectFill = 0.9;
constexpr float kPfRescaleLog2 = 8.0f;
// One exponential pair in NVKV_PF_POLY_EVERY runs on the FMA-pipe polynomial
// instead of MUFU ex2 (0: all on MUFU), balancing the two pipes.  Measured on
// the 8B prefill (16 x 1024, causal): 0 -> 207 us, 16 -> 208, 10 -> 202,
// 8 -> 197.5, 6 -> 199, 4 -> 204, 2 -> 217.
#ifndef NVKV_PF_POLY_EVERY
#define NVKV_PF_POLY_EVERY 8
#endif
constexpr int kPfPolyEvery = NVKV_PF_POLY_EVERY;  // rescale O only when the max grows by > 2^8

static_assert(kPfSmemBytes <= 232448, "prefill shared memory exceeds 227 KB");

struct PrefillParams {
  void* out;
  const uint32_t* cu_q;
  const uint32_t* cu_k;
  const uint32_t* block_tables;
  int64_t bt_stride;
  int64_t num_blocks;
  int num_q_heads;
  int group;
  int pair;  // 1: slots A/B are heads 2p, 2p+1 of one kv group; 0: slot A only
  int page_size;
  int num_q_tiles;
  int num_head_slots;  // hq / 2 with pairs, else hq
  // work plan (prefill_plan_kernel): plan[0] = q tiles in total, plan[1 + qt]
  // = sequences with more than qt q tiles; those sequences sorted by q-tile
  // count, most first: plan_seq[j] = {qs, q_len, ks, k_len}, plan_b[j] = b
  // (null: direct enumeration of num_q_tiles x num_head_slots x num_seqs
  // items, each checked against cu_seqlens)
  const uint32_t* plan;
  const uint4* plan_seq;
  const uint32_t* plan_b;
  int num_seqs;
  int max_k;           // max_seqlen_k: the block tables cover this many keys
  int64_t num_q_rows;  // rows of q and out
  int causal;
  float scale_log2;
  int* err;
};

// ---- tcgen05 wrappers -------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
#define NVKV_R32(r)                                                                          \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),    \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),      \
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),    \
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),    \
      "r"(r[29]), "r"(r[30]), "r"(r[31])
#define NVKV_W32(r)                                                                          \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),        \
      "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), \
      "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),          \
      "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),          \
      "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define NVKV_REGLIST                                                                           \
  "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24," \
  "%25,%26,%27,%28,%29,%30,%31}"
#define NVKV_REGLIST1                                                                          \
  "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24," \
  "%25,%26,%27,%28,%29,%30,%31,%32}"
// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 " NVKV_REGLIST ", [%32];"
               : NVKV_W32(r)
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], " NVKV_REGLIST1 ";" ::"r"(taddr),
               NVKV_R32(r)
               : "memory");
}

// 16 consecutive fp32 columns (used where the 128 S values are still live)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 2^x on the MUFU unit (PTX ex2.approx).
__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for two values on the FMA pipe: x = n + f with n = round(x), f in
// [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted here to the exact function
// (max relative error 7.5e-5, far below bf16's 2^-9 half-ulp); 2^n is added
// into the exponent bits.  The adds and FMAs are issued as packed f32x2
// pairs.  Valid for x in [-125, 126]; smaller x is clamped (the result,
// ~2^-125, is negligible next to the row sum it joins); NaN inputs clamp too.
__device__ __forceinline__ float2 ex2_poly2(float x0, float x1);
// max(a, b, c) in one instruction (three-input PTX max.f32; NaN handling as
// fmaxf: a NaN operand is ignored).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed two-lane f32 arithmetic (PTX add/fma .f32x2, sm_100): one
// instruction for two values on the FMA pipe.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// D (+)= A.B with A read from tensor memory (the P tile), B from shared memory.
__device__ __forceinline__ void tc_mma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float2 ex2_poly2(float x0, float x1) {
  const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const uint64_t x = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = f2_add(x, magic);  // t's low mantissa bits hold round(x)
  const float2 tv = f2_unpack(t);
  const uint64_t f = f2_sub(x, f2_sub(t, magic));
  uint64_t q = f2_fma(f2_pack(0.05517153f, 0.05517153f), f, f2_pack(0.24261111f, 0.24261111f));
  q = f2_fma(q, f, f2_pack(0.69326103f, 0.69326103f));
  q = f2_fma(q, f, f2_pack(0.99992806f, 0.99992806f));
  const float2 qv = f2_unpack(q);
  const int n0 = __float_as_int(tv.x) - 0x4B400000, n1 = __float_as_int(tv.y) - 0x4B400000;
  return make_float2(__int_as_float(__float_as_int(qv.x) + (n0 << 23)),
                     __int_as_float(__float_as_int(qv.y) + (n1 << 23)));
}
// Shared-memory matrix descriptor, SWIZZLE_128B, sm100 version bit.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: kind::f16, fp32 accumulate, M = N = 128.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_fmt, uint32_t b_mn_major) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (b_mn_major << 16) |
         ((uint32_t)(kPfBN >> 3) << 17) | ((uint32_t)(kPfBM >> 4) << 24);
}

// Two P values -> one packed 16-bit pair (cvt.rn.*x2.f32, round to nearest
// even).  A byte-permute packing on the ALU was measured slower (271 vs
// 264 us on the 8B prefill) once the exponentials moved to MUFU.
template <typename T>
__device__ __forceinline__ uint32_t pack_p(float a, float b) {
  return DT<T>::from_f2(a, b);
}

// P for one 64-key half of a row: e = 2^(s*scale - m) (masked keys -> 0) on
// the MUFU unit, packed in pairs into pk[32] (the half's 32 TMEM columns of
// 16-bit pairs); returns the sum of the e values.
template <typename T, bool kMask>
__device__ __forceinline__ float pf_exp_half(const float* sv, int kbase, int lim, float scale_log2,
                                             float m_use, uint32_t* pk) {
  uint64_t rs2 = f2_pack(0.f, 0.f);  // the row sum in two packed lanes
  const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_use, -m_use);
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    const float2 xx = f2_unpack(f2_fma(f2_pack(sv[i], sv[i + 1]), sc2, nm2));
    float e0, e1;
    if (kPfPolyEvery > 0 && (i / 2) % (kPfPolyEvery > 0 ? kPfPolyEvery : 1) == kPfPolyEvery - 1) {
      const float2 ee = ex2_poly2(xx.x, xx.y);  // this pair on the FMA pipe
      e0 = ee.x;
      e1 = ee.y;
    } else {
      e0 = ex2_mufu(xx.x);
      e1 = ex2_mufu(xx.y);
    }
    if (kMask) {
      e0 = kbase + i <= lim ? e0 : 0.f;
      e1 = kbase + i + 1 <= lim ? e1 : 0.f;
    }
    rs2 = f2_add(rs2, f2_pack(e0, e1));
    pk[i >> 1] = pack_p<T>(e0, e1);
  }
  const float2 rs = f2_unpack(rs2);
  return rs.x + rs.y;
}

// S_x = Q_x . K^T over D = 128: 8 MMAs of K = 16, advancing 32 bytes inside
// the 128-byte swizzle atom (both operands K-major, SWIZZLE_128B).
__device__ __forceinline__ void pf_issue_s(uint32_t d_tmem, uint32_t sq, uint32_t sk,
                                           uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < kPfD / 16; ++kk) {
    const uint32_t o = (kk >> 2) * kPfHalf + (kk & 3) * 32;
    tc_mma(d_tmem, sdesc(sq + o, 16, 1024), sdesc(sk + o, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}
// O_x (+)= P_x . V over 128 keys: P_x in TMEM (lane = query row, 64 columns of
// 16-bit key pairs over the S_x columns), 16 keys = 8 columns per MMA; V
// MN-major in shared memory (D contiguous, the two 64-wide D halves kPfHalf
// apart = LBO, 8 keys = SBO).
__device__ __forceinline__ void pf_issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t sv,
                                            uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kPfBN / 16; ++kk) {
    const uint64_t bd = sdesc(sv + kk * 16 * 128, kPfHalf, 1024);
    tc_mma_tmem_a(d_tmem, p_tmem + kk * 8, bd, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// ---- work plan --------------------------------------------------------------
// Checks one sequence's lengths against the buffers before anything is read
// or written for it.  Returns its q tiles, 0 for a decode row (q_len <= 1,
// the decode kernel's) and 0 for a malformed sequence: k_len < q_len, k_len
// > max_seqlen_k (its block-table row covers only max_seqlen_k keys) or rows
// qs .. qs + q_len past the q/out buffers.  q_len > max_seqlen_q is clamped
// to num_q_tiles.  With `err`, every malformed case is recorded as
// NVKV_DEVERR_SEQLEN.
__device__ __forceinline__ int pf_check_seq(uint32_t qs, int q_len, int k_len, int num_q_tiles,
                                            int max_k, int64_t num_q_rows, int* err) {
  if (q_len <= 1) return 0;
  if (k_len < q_len || k_len > max_k || (int64_t)qs + q_len > num_q_rows) {
    if (err) record_error(err, NVKV_DEVERR_SEQLEN);
    return 0;
  }
  const int n = (q_len + kPfBM - 1) / kPfBM;
  if (n > num_q_tiles) {
    if (err) record_error(err, NVKV_DEVERR_SEQLEN);
    return num_q_tiles;
  }
  return n;
}
__device__ __forceinline__ int pf_seq_tiles(const uint32_t* cu_q, const uint32_t* cu_k, int b,
                                            int num_q_tiles, int max_k, int64_t num_q_rows,
                                            int* err) {
  const uint32_t qs = cu_q[b];
  return pf_check_seq(qs, (int)(cu_q[b + 1] - qs), (int)(cu_k[b + 1] - cu_k[b]), num_q_tiles,
                      max_k, num_q_rows, err);
}

// Block-wide exclusive scan over 1024 threads; *total gets the sum.
__device__ __forceinline__ uint32_t pf_block_excl_scan(uint32_t v, uint32_t* part,
                                                       uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += t;
  }
  if (lane == 31) part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t pv = part[lane];
    uint32_t pi = pv;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, pi, d);
      if (lane >= d) pi += t;
    }
    part[lane] = pi - pv;
    if (lane == 31) *total = pi;
  }
  __syncthreads();
  return part[warp] + incl - v;
}

// One CTA of 1024 threads: a counting sort of the prefill sequences by their
// q-tile count (most first) into the plan, so the prefill kernel enumerates
// exactly its work items, however many decode rows share the batch.  Within
// one count the order follows the atomics; each item's arithmetic does not
// depend on which CTA takes it, so outputs do not change with that order.
// Plan layout: the counts, then (16-byte aligned) the records, then the ids.
__host__ __device__ inline size_t pf_plan_seq_word(int num_q_tiles) {
  return ((size_t)num_q_tiles + 1 + 3) & ~size_t(3);
}

__global__ void __launch_bounds__(1024)
    prefill_plan_kernel(const uint32_t* cu_q, const uint32_t* cu_k, int num_seqs,
                        int num_q_tiles, int max_k, int64_t num_q_rows, uint32_t* plan,
                        int* err) {
  pdl_launch_dependents();  // the prefill grid may start its prologue now
  extern __shared__ uint32_t hist[];  // [num_q_tiles + 1]: sequences per count, then cursors
  __shared__ uint32_t part[32], total, tiles;
  const int tid = threadIdx.x, Q = num_q_tiles;
  for (int i = tid; i <= Q; i += 1024) hist[i] = 0;
  if (tid == 0) tiles = 0;
  __syncthreads();
  for (int b = tid; b < num_seqs; b += 1024) {
    const int n = pf_seq_tiles(cu_q, cu_k, b, Q, max_k, num_q_rows, err);
    if (n > 0) {
      atomicAdd(&hist[n], 1u);
      atomicAdd(&tiles, (uint32_t)n);
    }
  }
  __syncthreads();
  // start[n] = sequences with more than n tiles: an exclusive scan over the
  // counts in descending order (entry i of the scan is count Q - i), one
  // contiguous chunk of it per thread
  const int per = (Q + 1 + 1023) / 1024;
  const int lo = tid * per, hi = min(lo + per, Q + 1);
  uint32_t sum = 0;
  for (int i = lo; i < hi; ++i) sum += hist[Q - i];
  uint32_t run = pf_block_excl_scan(sum, part, &total);
  for (int i = lo; i < hi; ++i) {
    const int n = Q - i;
    const uint32_t h = hist[n];
    hist[n] = run;  // becomes the scatter cursor of count n
    if (n < Q) plan[1 + n] = run;
    run += h;
  }
  if (tid == 0) plan[0] = tiles;
  __syncthreads();
  uint4* seq = reinterpret_cast<uint4*>(plan + pf_plan_seq_word(Q));
  uint32_t* ids = reinterpret_cast<uint32_t*>(seq + num_seqs);
  for (int b = tid; b < num_seqs; b += 1024) {
    const int n = pf_seq_tiles(cu_q, cu_k, b, Q, max_k, num_q_rows, nullptr);
    if (n > 0) {
      const uint32_t pos = atomicAdd(&hist[n], 1u);
      const uint32_t qs = cu_q[b], ks = cu_k[b];
      seq[pos] = make_uint4(qs, cu_q[b + 1] - qs, ks, cu_k[b + 1] - ks);
      ids[pos] = (uint32_t)b;
    }
  }
}

// One work item = (q tile, head pair / head, sequence).  Items run level by
// level from the last q tile down (the heaviest causal tiles first); level qt
// holds plan[1 + qt] sequences x num_head_slots, the head slot varying
// fastest.  The level of item w is found by walking the (few, L1-resident)
// level counts from the top on every call: nothing stays live across the
// roles' tile loops, whose softmax warps are at the register limit.
struct PfItem {
  int b, head0, kvh, i0, q_len, k_len, off, ntiles;
  uint32_t qs, ks;
};
template <bool kPlan>
__device__ __forceinline__ int pf_num_items(const PrefillParams& p) {
  return kPlan ? (int)__ldg(p.plan) * p.num_head_slots
               : p.num_q_tiles * p.num_head_slots * p.num_seqs;
}
// Direct enumeration: the same level order with every sequence in each level;
// returns false for an empty item (a decode row, a tile past q_len, or a
// malformed sequence, which pf_check_seq reports).
__device__ __forceinline__ bool pf_item_direct(const PrefillParams& p, int w, PfItem& it) {
  const int per_tile = p.num_head_slots * p.num_seqs;
  const int qt = p.num_q_tiles - 1 - w / per_tile;
  const int rem = w % per_tile;
  const int y = rem % p.num_head_slots;
  it.b = rem / p.num_head_slots;
  it.head0 = p.pair ? 2 * y : y;
  it.kvh = it.head0 / p.group;
  it.qs = __ldg(p.cu_q + it.b);
  it.q_len = (int)(__ldg(p.cu_q + it.b + 1) - it.qs);
  it.i0 = qt * kPfBM;
  if (it.q_len <= 1 || it.i0 >= it.q_len) return false;
  it.ks = __ldg(p.cu_k + it.b);
  it.k_len = (int)(__ldg(p.cu_k + it.b + 1) - it.ks);
  it.off = it.k_len - it.q_len;
  // every item of a sequence is checked; the items of q tile 0 (which every
  // prompt has) report, once per head slot
  if (pf_check_seq(it.qs, it.q_len, it.k_len, p.num_q_tiles, p.max_k, p.num_q_rows,
                   qt == 0 ? p.err : nullptr) == 0)
    return false;
  const int last_row = min(it.i0 + kPfBM, it.q_len) - 1;
  const int kmax = p.causal ? min(it.k_len, last_row + it.off + 1) : it.k_len;
  it.ntiles = (kmax + kPfBN - 1) / kPfBN;
  return true;
}
template <bool kPlan>
__device__ __forceinline__ bool pf_item(const PrefillParams& p, int w, PfItem& it) {
  if (!kPlan) return pf_item_direct(p, w, it);
  int qt = p.num_q_tiles - 1, base = 0;
  for (; qt >= 0; --qt) {
    const int n = (int)__ldg(p.plan + 1 + qt) * p.num_head_slots;
    if (w < base + n) break;
    base += n;
  }
  if (qt < 0) return false;
  const int r = w - base;
  const int y = r % p.num_head_slots, j = r / p.num_head_slots;
  const uint4 e = __ldg(p.plan_seq + j);
  it.b = (int)__ldg(p.plan_b + j);
  it.head0 = p.pair ? 2 * y : y;
  it.kvh = it.head0 / p.group;
  it.qs = e.x;
  it.q_len = (int)e.y;
  it.i0 = qt * kPfBM;
  it.ks = e.z;
  it.k_len = (int)e.w;
  it.off = it.k_len - it.q_len;
  const int last_row = min(it.i0 + kPfBM, it.q_len) - 1;
  const int kmax = p.causal ? min(it.k_len, last_row + it.off + 1) : it.k_len;
  it.ntiles = (kmax + kPfBN - 1) / kPfBN;
  return true;
}

// Item of round k for this CTA: rounds alternate direction (snake order), so
// the CTA that took a round's heaviest item takes the next round's lightest.
__device__ __forceinline__ int pf_work(int k) {
  const int c = (k & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
  return k * (int)gridDim.x + c;
}

// Persistent: one CTA per SM walks its items with the barriers, TMEM and
// descriptors set up once.  Every barrier phase is a running count over the
// CTA's items (g = key tiles so far per slot, t = K/V ring loads, nq =
// items), so the MMA warp issues item i+1's first S while the softmax warps
// still run item i's epilogue, and the producer loads item i+1's Q as soon as
// item i's last S MMA has read Q (q_empty).  O_x needs no extra barrier: its
// next overwrite (item i+1's first PV, accumulate = 0) waits on p_full, which
// the softmax warps arrive only after their epilogue has read O_x.
template <typename T, bool kPlan>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPfOffBar);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;             // the item's last S MMA has read Q
  uint64_t* kv_full = bars + 2;             // [kPfSlots]
  uint64_t* kv_empty = kv_full + kPfSlots;  // [kPfSlots]
  uint64_t* s_full = kv_empty + kPfSlots;   // [2]: S_x written by the MMA
  uint64_t* p_full = s_full + 2;            // [2]: S_x read, P_x written (O_x rescaled / read)
  uint64_t* o_done = p_full + 2;            // [2]: PV_x finished (O_x stable, P_x free)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nslot = p.pair ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kPfSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 128);
      mbar_init(&o_done[x], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kPfTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the work plan (and the inputs) of the kernels before this one

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      uint32_t nq = 0, t = 0;  // items loaded, K/V ring loads (running over items)
      bool ok = true;
      for (int k = 0; ok && (int64_t)k * gridDim.x < pf_num_items<kPlan>(p); ++k) {
        const int w = pf_work(k);
        PfItem it;
        if (w >= pf_num_items<kPlan>(p) || !pf_item<kPlan>(p, w, it)) continue;
        if (nq > 0 && !mbar_wait(q_empty, (nq - 1) & 1u, p.err)) break;
        mbar_arrive_expect_tx(q_full, nslot * kPfTile);
        for (int x = 0; x < nslot; ++x) {
          uint8_t* qd = smem + (x ? kPfOffQB : kPfOffQA);
          tma_load_3d(qd, &tmap_q, q_full, 0, it.head0 + x, (int)(it.qs + it.i0));
          tma_load_3d(qd + kPfHalf, &tmap_q, q_full, 64, it.head0 + x, (int)(it.qs + it.i0));
        }
        ++nq;
        for (int u = 0; u < 2 * it.ntiles; ++u, ++t) {  // K_0, V_0, K_1, V_1, ...
          const int j = u >> 1;
          const int s = (int)(t % kPfSlots);
          const uint32_t ph = (t / kPfSlots) & 1u;
          if (t >= kPfSlots && !mbar_wait(&kv_empty[s], ph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          const int j0 = j * kPfBN;
          int64_t row;
          if (p.block_tables) {
            uint32_t page = p.block_tables[(int64_t)it.b * p.bt_stride + j0 / p.page_size];
            if ((int64_t)page >= p.num_blocks) {
              record_error(p.err, NVKV_DEVERR_BLOCK_RANGE);
              page = 0;
            }
            row = (int64_t)page * p.page_size + (j0 % p.page_size);
          } else {
            row = (int64_t)it.ks + j0;
          }
          uint8_t* dst = smem + kPfOffKV + s * kPfTile;
          const CUtensorMap* map = (u & 1) ? &tmap_v : &tmap_k;
          mbar_arrive_expect_tx(&kv_full[s], kPfTile);
          tma_load_3d(dst, map, &kv_full[s], 0, it.kvh, (int)row);
          tma_load_3d(dst + kPfHalf, map, &kv_full[s], 64, it.kvh, (int)row);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_qk = make_idesc(fmt, 0u);
      constexpr uint32_t idesc_pv = make_idesc(fmt, 1u);
      const uint32_t kv0 = smem_u32(smem + kPfOffKV);
      const uint32_t sqa = smem_u32(smem + kPfOffQA), sqb = smem_u32(smem + kPfOffQB);
#define PF_SLOT(t) (kv0 + (uint32_t)((t) % kPfSlots) * kPfTile)
#define PF_PAR(t) ((uint32_t)((t) / kPfSlots) & 1u)
#define PF_FULL(t) (&kv_full[(t) % kPfSlots])
      uint32_t nq = 0, t = 0, g = 0;  // items, K/V ring position, key tiles per slot
      bool ok = true;
      for (int k = 0; ok && (int64_t)k * gridDim.x < pf_num_items<kPlan>(p); ++k) {
        const int w = pf_work(k);
        PfItem it;
        if (w >= pf_num_items<kPlan>(p) || !pf_item<kPlan>(p, w, it)) continue;
        const int n = it.ntiles;
        // S_x(g) of the item's first key tile: Q and K_0 (S_x / P_x(g - 1) were
        // consumed by PV_x(g - 1), issued before it on the in-order pipe)
        ok = mbar_wait(q_full, nq & 1u, p.err) && mbar_wait(PF_FULL(t), PF_PAR(t), p.err);
        if (!ok) break;
        tc_fence_after();
        pf_issue_s(tmem + 0u, sqa, PF_SLOT(t), idesc_qk);
        tc_commit(&s_full[0]);
        if (p.pair) {
          pf_issue_s(tmem + 128u, sqb, PF_SLOT(t), idesc_qk);
          tc_commit(&s_full[1]);
        }
        tc_commit(&kv_empty[t % kPfSlots]);
        if (n == 1) tc_commit(q_empty);
        ++nq;
        for (int j = 0; j < n; ++j, ++g) {
          const uint32_t pj = g & 1u;
          const bool more = j + 1 < n;
          const uint32_t tv = t + 2 * j + 1, tk = t + 2 * j + 2;  // V_j, K_{j+1}
          ok = mbar_wait(PF_FULL(tv), PF_PAR(tv), p.err) && mbar_wait(&p_full[0], pj, p.err);
          if (!ok) break;
          tc_fence_after();
          pf_issue_pv(tmem + 256u, tmem + 0u, PF_SLOT(tv), idesc_pv, j > 0);
          tc_commit(&o_done[0]);
          if (more) {
            ok = mbar_wait(PF_FULL(tk), PF_PAR(tk), p.err);
            if (!ok) break;
            tc_fence_after();
            pf_issue_s(tmem + 0u, sqa, PF_SLOT(tk), idesc_qk);
            tc_commit(&s_full[0]);
          }
          if (p.pair) {
            ok = mbar_wait(&p_full[1], pj, p.err);
            if (!ok) break;
            tc_fence_after();
            pf_issue_pv(tmem + 384u, tmem + 128u, PF_SLOT(tv), idesc_pv, j > 0);
            tc_commit(&o_done[1]);
          }
          tc_commit(&kv_empty[tv % kPfSlots]);  // V_j: both P.V issued
          if (more) {
            if (p.pair) {
              pf_issue_s(tmem + 128u, sqb, PF_SLOT(tk), idesc_qk);
              tc_commit(&s_full[1]);
            }
            tc_commit(&kv_empty[tk % kPfSlots]);  // K_{j+1}: both S issued
            if (j + 2 == n) tc_commit(q_empty);   // the item's last S MMAs read Q
          }
        }
        t += 2 * (uint32_t)n;
      }
#undef PF_SLOT
#undef PF_PAR
#undef PF_FULL
    }
  } else {
    // ------------------------------ softmax warpgroups ------------------------------
    const int x = (warp - 2) >> 2;  // slot: warps 2-5 -> A, 6-9 -> B
    if (x < nslot) {
      const int quarter = warp & 3;  // TMEM lane quarter this warp may access
      const int r = quarter * 32 + lane;
      const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
      const uint32_t col_s = x ? 128u : 0u, col_o = x ? 384u : 256u;
      uint32_t g = 0;  // key tiles of this slot so far (running over items)
      bool alive = true;
      for (int k = 0; alive && (int64_t)k * gridDim.x < pf_num_items<kPlan>(p); ++k) {
        const int w = pf_work(k);
        PfItem it;
        if (w >= pf_num_items<kPlan>(p) || !pf_item<kPlan>(p, w, it)) continue;
        const int qi = it.i0 + r;
        const int lim_row = p.causal ? min(it.k_len - 1, qi + it.off) : it.k_len - 1;
        float m_ref = -INFINITY, l = 0.f;
        for (int j = 0; j < it.ntiles; ++j, ++g) {
          const uint32_t pj = g & 1u;
          // decisions stay warp-uniform: the tcgen05.ld/st below are .sync.aligned.
          // s_full(g) also means PV_x(g - 1) is complete (it was issued before
          // S_x(g)): O_x is stable for a rescale.
          if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], pj, p.err))) {
            alive = false;
            break;
          }
          tc_fence_after();
          const int lim = lim_row - j * kPfBN;  // keys c <= lim are visible
          // the whole warp sees every key of this tile: no masking needed
          const bool vis = __all_sync(0xffffffffu, lim >= kPfBN - 1);
          // the whole S row in registers: one TMEM round trip, exact tile max
          float sv[128];
          tmem_ld32(lane_addr + col_s, sv);
          tmem_ld32(lane_addr + col_s + 32, sv + 32);
          tmem_ld32(lane_addr + col_s + 64, sv + 64);
          tmem_ld32(lane_addr + col_s + 96, sv + 96);
          tmem_wait_ld();
          // four independent max chains, then combined
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          if (vis) {
#pragma unroll
            for (int i = 0; i < 128; i += 2) m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], sv[i], sv[i + 1]);
          } else {
#pragma unroll
            for (int i = 0; i < 128; i += 2)
              m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], i <= lim ? sv[i] : -INFINITY,
                                       i + 1 <= lim ? sv[i + 1] : -INFINITY);
          }
          const float mx = fmaxf(fmax3(m4[0], m4[1], m4[2]), m4[3]);
          // keep the reference max unless the row max grew by more than 2^8
          // (exponentials stay <= 256); then the TMEM O row is rescaled below
          const float m_new = fmaxf(m_ref, mx * p.scale_log2);
          const bool need = m_new > m_ref + kPfRescaleLog2;
          const bool rescale = j >= 1 && __any_sync(0xffffffffu, need);
          const float fac = need ? exp2f(m_ref - m_new) : 1.f;
          if (j == 0 || need) m_ref = m_new;
          const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
          // P_x over the S_x columns just read: keys 0-63 -> columns 0-31,
          // keys 64-127 -> columns 32-63 (the PV MMA's A operand)
          float rs;
          {
            uint32_t pk[32];
            rs = vis ? pf_exp_half<T, false>(sv, 0, lim, p.scale_log2, m_use, pk)
                     : pf_exp_half<T, true>(sv, 0, lim, p.scale_log2, m_use, pk);
            tmem_st32(lane_addr + col_s, reinterpret_cast<const float*>(pk));
          }
          {
            uint32_t pk[32];
            rs += vis ? pf_exp_half<T, false>(sv + 64, 64, lim, p.scale_log2, m_use, pk)
                      : pf_exp_half<T, true>(sv + 64, 64, lim, p.scale_log2, m_use, pk);
            tmem_st32(lane_addr + col_s + 32, reinterpret_cast<const float*>(pk));
          }
          if (rescale) {  // O_x *= 2^(m_old - m_new) before PV_x(g) adds to it
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
              float o[16];
              tmem_ld16(lane_addr + col_o + c * 16, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] *= fac;
              tmem_st16(lane_addr + col_o + c * 16, o);
            }
            l *= fac;
          }
          tmem_wait_st();
          l += rs;
          tc_fence_before();
          mbar_arrive(&p_full[x]);
        }
        // the item's last PV_x: O_x complete
        if (!alive ||
            !__all_sync(0xffffffffu, mbar_wait(&o_done[x], (g - 1u) & 1u, p.err))) {
          alive = false;
          break;
        }
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* dst = reinterpret_cast<T*>(p.out) +
                 ((int64_t)(it.qs + qi) * p.num_q_heads + it.head0 + x) * kPfD;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(lane_addr + col_o + c * 32, o);
          tmem_wait_ld();
          if (qi < it.q_len) {
#pragma unroll
            for (int d = 0; d < 32; d += 8) {
              uint4 wv;
              wv.x = DT<T>::from_f2(o[d] * inv, o[d + 1] * inv);
              wv.y = DT<T>::from_f2(o[d + 2] * inv, o[d + 3] * inv);
              wv.z = DT<T>::from_f2(o[d + 4] * inv, o[d + 5] * inv);
              wv.w = DT<T>::from_f2(o[d + 6] * inv, o[d + 7] * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + d) = wv;
            }
          }
        }
        // O_x read (tcgen05.wait::ld above): the next item's first PV_x may
        // overwrite it once this warpgroup arrives on p_full
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, kPfTmemCols);
  }
}

// ---------------------------------------------------------------------------
size_t prefill_plan_bytes(int num_seqs, int max_seqlen_q) {
  if (max_seqlen_q <= 1 || num_seqs <= 0) return 0;
  const int q_tiles = (max_seqlen_q + kPfBM - 1) / kPfBM;
  const size_t words = pf_plan_seq_word(q_tiles) + 5 * (size_t)num_seqs;
  return (words * sizeof(uint32_t) + 255) & ~size_t(255);
}

template <typename T, bool kPlan>
static int launch_prefill_grid(dim3 grid, const CUtensorMap& mq, const CUtensorMap& mk,
                               const CUtensorMap& mv, const PrefillParams& p,
                               cudaStream_t stream) {
  auto kern = paged_prefill_kernel<T, kPlan>;
  static unsigned long long attr_done = 0;  // one per instantiation
  int rc = ensure_smem_attr((const void*)kern, kPfSmemBytes, &attr_done);
  if (rc) return rc;
  return launch_pdl(kern, grid, dim3(kPfThreads), kPfSmemBytes, stream, "paged prefill launch",
                    mq, mk, mv, p);
}

int launch_paged_prefill(const AttnArgs& a) {
  const int64_t rows = a.block_tables ? a.num_blocks * a.page : a.num_blocks;
  CUtensorMap mq, mk, mv;
  int rc = encode_kv_tensor_map(&mq, a.q, kPfD, a.hq, a.num_q_rows, a.q_stride * 2, 64, kPfBM,
                                true);
  if (rc) return rc;
  rc = encode_kv_tensor_map(&mk, a.k_cache, kPfD, a.hkv, rows, a.kv_stride * 2, 64, kPfBN, true);
  if (rc) return rc;
  rc = encode_kv_tensor_map(&mv, a.v_cache, kPfD, a.hkv, rows, a.kv_stride * 2, 64, kPfBN, true);
  if (rc) return rc;
  PrefillParams p;
  p.out = a.out;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.num_blocks = a.num_blocks;
  p.num_q_heads = a.hq;
  p.group = a.hq / a.hkv;
  p.pair = (p.group % 2 == 0) ? 1 : 0;  // two heads of one kv group per CTA
  p.page_size = a.page;
  p.num_q_tiles = (a.max_q + kPfBM - 1) / kPfBM;
  p.num_head_slots = p.pair ? a.hq / 2 : a.hq;
  const int64_t items = (int64_t)p.num_q_tiles * p.num_head_slots * a.num_seqs;  // upper bound
  if (items > INT32_MAX - kPfCtas || p.num_q_tiles > kPfMaxQTiles)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged prefill: too many tiles");
  if (items == 0) return NVKV_OK;
  const size_t plan_off =
      attention_plan_offset(decode_workspace_bytes(a.num_seqs, a.hq, a.hkv, a.max_k, a.fp8_layout));
  const size_t plan_need = prefill_plan_bytes(a.num_seqs, a.max_q);
  if (!a.ws || a.ws_bytes < plan_off + plan_need)
    return set_error(NVKV_ERR_WORKSPACE, "paged prefill: workspace too small for the work plan");
  // Empty candidates (decode rows, tiles past a short prompt) cost a skip and
  // leave holes in the balanced rounds; the plan removes them but costs a
  // launch in front of the grid.
  const int64_t cand_tiles = (int64_t)p.num_q_tiles * a.num_seqs;
  const bool use_plan = items > (int64_t)kPfCtas * kPfDirectItemsPerCta &&
                        (double)(a.num_q_rows / kPfBM) < kPfDirectFill * (double)cand_tiles;
  uint32_t* plan = use_plan ? reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.ws) + plan_off)
                            : nullptr;
  p.plan = plan;
  p.plan_seq = use_plan ? reinterpret_cast<const uint4*>(plan + pf_plan_seq_word(p.num_q_tiles))
                        : nullptr;
  p.plan_b = use_plan ? reinterpret_cast<const uint32_t*>(p.plan_seq + a.num_seqs) : nullptr;
  p.num_seqs = a.num_seqs;
  p.max_k = a.max_k;
  p.num_q_rows = a.num_q_rows;
  p.causal = a.causal;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = device_error_word();
  if (use_plan) {
    prefill_plan_kernel<<<1, 1024, (p.num_q_tiles + 1) * sizeof(uint32_t), a.stream>>>(
        a.cu_q, a.cu_k, a.num_seqs, p.num_q_tiles, a.max_k, a.num_q_rows, plan, p.err);
    rc = check_cuda(cudaGetLastError(), "prefill plan launch");
    if (rc) return rc;
  }
  // one persistent CTA per SM (the shared-memory footprint allows one)
  const dim3 grid((unsigned)std::min<int64_t>(items, kPfCtas));
  if (a.dtype == NVKV_DTYPE_BF16)
    rc = use_plan ? launch_prefill_grid<__nv_bfloat16, true>(grid, mq, mk, mv, p, a.stream)
                  : launch_prefill_grid<__nv_bfloat16, false>(grid, mq, mk, mv, p, a.stream);
  else
    rc = use_plan ? launch_prefill_grid<__half, true>(grid, mq, mk, mv, p, a.stream)
                  : launch_prefill_grid<__half, false>(grid, mq, mk, mv, p, a.stream);
  return rc;
}

}  // namespace nvkv
