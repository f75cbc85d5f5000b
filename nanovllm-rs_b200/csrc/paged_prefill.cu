// Kernel 3: varlen (paged) causal prefill attention on tcgen05 tensor cores.
//
// Replaces the prefill / mixed-batch uses of candle_flash_attn
// (flash_attn_varlen and flash_attn_varlen_paged_windowed, nanovllm_rs/src/
// layers/attention.rs:43-73; FA2 with SM80 mma.sync) for every sequence
// whose q_len > 1 (q_len == 1 rows run on the decode kernel).
//
// One CTA = 128 query rows of one query head of one sequence.  6 warps:
//   warp 0      TMA producer: Q tile once, then K/V tiles of 128 keys
//               (pages resolved through block_tables) into a 2-stage ring,
//               SWIZZLE_128B, each CTA loading its own tiles;
//   warp 1      allocates 512 TMEM columns and issues every tcgen05.mma from
//               one thread: S_j = Q.K_j^T (K-major A and B, M=N=128, K=16 x 8)
//               into a double-buffered S in TMEM, then O_j = P_j.V_j (P K-major
//               from shared memory, V MN-major) into a TMEM O tile;
//               tcgen05.commit signals the mbarriers;
//   warps 2-5   softmax warpgroup: thread r owns query row r (TMEM lane r).
//               Per key tile it reads its S row from TMEM (tcgen05.ld
//               32x32b), applies the causal / length mask (bottom-right
//               aligned: key j visible to query i iff j <= i + k_len - q_len),
//               runs the fp32 online softmax, writes P (bf16/f16) into the
//               swizzled shared-memory tile the next MMA reads, and folds the
//               previous O tile into a 128-float register accumulator.
// Roofline: tensor cores; flops = 4 * D * (visible (query, key) pairs).
#include <type_traits>

#include "common.cuh"

namespace nvkv {

constexpr int kPfD = 128;
constexpr int kPfBM = 128;
constexpr int kPfBN = 128;
constexpr int kPfStages = 2;
constexpr int kPfThreads = 6 * 32;
constexpr int kPfHalf = 128 * 128;          // 128 rows x 128 B (64 elements)
constexpr int kPfTile = 2 * kPfHalf;        // 32 KB: 128 rows x 128 elements
constexpr int kPfOffQ = 0;
constexpr int kPfOffK = kPfOffQ + kPfTile;
constexpr int kPfOffV = kPfOffK + kPfStages * kPfTile;
constexpr int kPfOffP = kPfOffV + kPfStages * kPfTile;
constexpr int kPfOffBar = kPfOffP + kPfTile;
constexpr int kPfNumBars = 1 + 3 * kPfStages + 2 + 2 + 1 + 1;
constexpr int kPfSmemBytes = kPfOffBar + kPfNumBars * 8 + 16 + 1024;
constexpr uint32_t kPfTmemCols = 512;
constexpr uint32_t kPfColS0 = 0, kPfColS1 = 128, kPfColO = 256;

struct PrefillParams {
  void* out;
  const uint32_t* cu_q;
  const uint32_t* cu_k;
  const uint32_t* block_tables;
  int64_t bt_stride;
  int64_t num_blocks;
  int num_q_heads;
  int group;
  int page_size;
  int num_q_tiles;
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
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
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

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPfOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kPfStages;
  uint64_t* kv_empty = v_full + kPfStages;
  uint64_t* s_full = kv_empty + kPfStages;  // [2]
  uint64_t* s_free = s_full + 2;            // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* o_full = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);

  const int qt = p.num_q_tiles - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int hq = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t qs = p.cu_q[b];
  const int q_len = (int)(p.cu_q[b + 1] - qs);
  if (q_len <= 1) return;  // q_len == 1 rows belong to the decode kernel
  const int i0 = qt * kPfBM;
  if (i0 >= q_len) return;
  const uint32_t ks = p.cu_k[b];
  const int k_len = (int)(p.cu_k[b + 1] - ks);
  const int off = k_len - q_len;
  if (off < 0) {
    if (threadIdx.x == 0) record_error(p.err, NVKV_DEVERR_SEQLEN);
    return;
  }
  const int last_row = min(i0 + kPfBM, q_len) - 1;
  const int kmax = p.causal ? min(k_len, last_row + off + 1) : k_len;
  const int ntiles = (kmax + kPfBN - 1) / kPfBN;
  const int kvh = hq / p.group;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
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

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      mbar_arrive_expect_tx(q_full, kPfTile);
      tma_load_3d(smem + kPfOffQ, &tmap_q, q_full, 0, hq, (int)(qs + i0));
      tma_load_3d(smem + kPfOffQ + kPfHalf, &tmap_q, q_full, 64, hq, (int)(qs + i0));
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kPfStages;
        const uint32_t ph = (uint32_t)(j / kPfStages) & 1u;
        if (j >= kPfStages && !mbar_wait(&kv_empty[st], ph ^ 1u, p.err)) break;
        const int j0 = j * kPfBN;
        int64_t row;
        if (p.block_tables) {
          uint32_t page = p.block_tables[(int64_t)b * p.bt_stride + j0 / p.page_size];
          if ((int64_t)page >= p.num_blocks) {
            record_error(p.err, NVKV_DEVERR_BLOCK_RANGE);
            page = 0;
          }
          row = (int64_t)page * p.page_size + (j0 % p.page_size);
        } else {
          row = (int64_t)ks + j0;
        }
        uint8_t* kd = smem + kPfOffK + st * kPfTile;
        uint8_t* vd = smem + kPfOffV + st * kPfTile;
        mbar_arrive_expect_tx(&k_full[st], kPfTile);
        tma_load_3d(kd, &tmap_k, &k_full[st], 0, kvh, (int)row);
        tma_load_3d(kd + kPfHalf, &tmap_k, &k_full[st], 64, kvh, (int)row);
        mbar_arrive_expect_tx(&v_full[st], kPfTile);
        tma_load_3d(vd, &tmap_v, &v_full[st], 0, kvh, (int)row);
        tma_load_3d(vd + kPfHalf, &tmap_v, &v_full[st], 64, kvh, (int)row);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_qk = make_idesc(fmt, 0u);
      constexpr uint32_t idesc_pv = make_idesc(fmt, 1u);
      const uint32_t sq = smem_u32(smem + kPfOffQ);
      const uint32_t sp = smem_u32(smem + kPfOffP);
      bool ok = mbar_wait(q_full, 0, p.err);
      auto issue_pv = [&](int j) {
        const int st = j % kPfStages;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, p.err)) return false;
        if (!mbar_wait(&v_full[st], (uint32_t)(j / kPfStages) & 1u, p.err)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + kPfOffV + st * kPfTile);
#pragma unroll
        for (int kk = 0; kk < kPfBN / 16; ++kk) {
          // A = P (K-major over keys): half kk/4, +32 B per 16 keys inside the half
          const uint64_t ad = sdesc(sp + (kk >> 2) * kPfHalf + (kk & 3) * 32, 16, 1024);
          // B = V (MN-major over D): 16 keys = 16 rows of 128 B; D halves LBO apart
          const uint64_t bd = sdesc(sv + kk * 16 * 128, kPfHalf, 1024);
          tc_mma(tmem + kPfColO, ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        tc_commit(o_full);
        tc_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % kPfStages;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], (uint32_t)(j / kPfStages) & 1u, p.err)) break;
        if (j >= 2 && !mbar_wait(&s_free[sb], ((uint32_t)(j >> 1) & 1u) ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + kPfOffK + st * kPfTile);
        const uint32_t dcol = sb ? kPfColS1 : kPfColS0;
#pragma unroll
        for (int kk = 0; kk < kPfD / 16; ++kk) {
          const uint32_t o = (kk >> 2) * kPfHalf + (kk & 3) * 32;
          tc_mma(tmem + dcol, sdesc(sq + o, 16, 1024), sdesc(sk + o, 16, 1024), idesc_qk,
                 kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && ntiles > 0) issue_pv(ntiles - 1);
    }
  } else {
    // ------------------------------ softmax warpgroup ------------------------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const int qi = i0 + r;
    const int lim_row = p.causal ? min(k_len - 1, qi + off) : k_len - 1;
    uint8_t* pbase = smem + kPfOffP;

    float acc[kPfD];
#pragma unroll
    for (int d = 0; d < kPfD; ++d) acc[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool alive = true;

    for (int j = 0; j < ntiles && alive; ++j) {
      const int sb = j & 1;
      // decisions stay warp-uniform: tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (uint32_t)(j >> 1) & 1u, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = lane_addr + (sb ? kPfColS1 : kPfColS0);
      const int lim = lim_row - j * kPfBN;  // visible keys of this tile: c <= lim
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(scol + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, (c * 32 + i) <= lim ? v[i] : -INFINITY);
      }
      const float m_new = fmaxf(m, mx * p.scale_log2);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      // fold the previous O tile (its MMA also released the P buffer)
      if (j >= 1) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_full, (uint32_t)(j - 1) & 1u, p.err))) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(lane_addr + kPfColO + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[c * 32 + i] = acc[c * 32 + i] * alpha_prev + v[i];
        }
      }
      // pass 2: P = exp2(s*scale - m) -> swizzled K-major tile in shared memory
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(scol + c * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float e0 = (c * 32 + i) <= lim ? exp2f(v[i] * p.scale_log2 - m_use) : 0.f;
          const float e1 = (c * 32 + i + 1) <= lim ? exp2f(v[i + 1] * p.scale_log2 - m_use) : 0.f;
          rs += e0 + e1;
          pk[i >> 1] = DT<T>::from_f2(e0, e1);
        }
        uint8_t* half = pbase + (c >> 1) * kPfHalf;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t chunk = (uint32_t)((c & 1) * 4 + u);
          uint4* dst = reinterpret_cast<uint4*>(half + sw128_offset((uint32_t)r, chunk));
          *dst = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
      l = l * alpha + rs;
      m = m_new;
      alpha_prev = alpha;
    }
    if (alive && ntiles > 0) {
      if (__all_sync(0xffffffffu, mbar_wait(o_full, (uint32_t)(ntiles - 1) & 1u, p.err))) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(lane_addr + kPfColO + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[c * 32 + i] = acc[c * 32 + i] * alpha_prev + v[i];
        }
      }
    }
    if (qi < q_len) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)(qs + qi) * p.num_q_heads + hq) * kPfD;
#pragma unroll
      for (int d = 0; d < kPfD; d += 8) {
        uint4 w;
        w.x = DT<T>::from_f2(acc[d] * inv, acc[d + 1] * inv);
        w.y = DT<T>::from_f2(acc[d + 2] * inv, acc[d + 3] * inv);
        w.z = DT<T>::from_f2(acc[d + 4] * inv, acc[d + 5] * inv);
        w.w = DT<T>::from_f2(acc[d + 6] * inv, acc[d + 7] * inv);
        *reinterpret_cast<uint4*>(dst + d) = w;
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
  p.page_size = a.page;
  p.num_q_tiles = (a.max_q + kPfBM - 1) / kPfBM;
  p.causal = a.causal;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = device_error_word();
  dim3 grid(p.num_q_tiles, a.hq, a.num_seqs);
  if (a.dtype == NVKV_DTYPE_BF16) {
    auto kern = paged_prefill_kernel<__nv_bfloat16>;
    static unsigned long long attr_done_1 = 0;
    rc = ensure_smem_attr((const void*)kern, kPfSmemBytes, &attr_done_1);
    if (rc) return rc;
    kern<<<grid, kPfThreads, kPfSmemBytes, a.stream>>>(mq, mk, mv, p);
  } else {
    auto kern = paged_prefill_kernel<__half>;
    static unsigned long long attr_done_2 = 0;
    rc = ensure_smem_attr((const void*)kern, kPfSmemBytes, &attr_done_2);
    if (rc) return rc;
    kern<<<grid, kPfThreads, kPfSmemBytes, a.stream>>>(mq, mk, mv, p);
  }
  return check_cuda(cudaGetLastError(), "paged prefill launch");
}

}  // namespace nvkv
