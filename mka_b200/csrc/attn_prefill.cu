// Causal flash-attention forward (prefill) on tcgen05 tensor cores, head_dim 128,
// GQA, bottom-right causal alignment (query i sees keys <= i + Tk - Tq), with the
// log-sum-exp of every row as a second output.
//
// Reference semantics: the causal attention of the FastMKA forward
// (F.scaled_dot_product_attention at mka/layers/fastmka.py:134,157 and
// mka/hf/attention.py:142; the explicit masked softmax at fastmka.py:166-174 and
// hf/attention.py:188-193; fastmka_attn at mka/cuda/fastmka_attn.cu:51-131, which
// uses the same Tk - Tq causal offset). GQA is handled by indexing the shared
// K/V head instead of materialising _repeat_kv (hf/attention.py:28-33,128-129).
//
// One CTA per (128-query tile, query head). Warp roles:
//   warp 0      TMA producer: Q once, then K and V tiles (128 keys) into a
//               two-stage shared-memory ring (128-byte swizzle)
//   warp 1      MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers; then
//               O += P_{j-1} V_{j-1} with P read straight from TMEM
//   warp 2      TMEM allocator (512 columns: S0 | S1 | O)
//   warps 4..7  softmax: thread i owns query row i; reads its S row from TMEM,
//               applies the causal mask on diagonal tiles, keeps the running
//               max m and sum z (online softmax), writes P as packed bf16 back
//               over S, rescales O in TMEM only when the max grew by more than
//               2^8 (exact: the final 1/z uses the same stale max), and at the
//               end normalises O and writes O and LSE.
// KV tiles past the causal limit of the query tile are never loaded.
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kHeadDim = 128;
constexpr int kKS = 2;
constexpr int kThreads = 256;
constexpr int kTileBytes = 128 * 128 * 2;  // 32 KB
constexpr int kHalfBytes = kTileBytes / 2;  // one 64-column swizzle box
constexpr int kSmemBytes = kTileBytes * (1 + 2 * kKS) + 1024 + 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct AttnParams {
  int B, Hq, Hkv, Tq, Tk;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;  // O[b, t, h, :]
  int64_t o_sb, o_st, o_sh;
  float* lse;        // lse[b, h, t] (may be null)
  int64_t lse_sb, lse_sh;
  int n_qtiles;
  uint32_t* status;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;
  uint8_t* sV = sK + kKS * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKS * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kKS;
  uint64_t* v_full = k_empty + kKS;
  uint64_t* v_empty = v_full + kKS;
  uint64_t* s_full = v_empty + kKS;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_bar = p_full + 2;   // [2]: PV_i completes pv_bar[i & 1]
  uint64_t* o_full = pv_bar + 2;   // the last PV has completed
  uint64_t* mma_done = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  // ---- tile coordinates: the G query heads of one KV head are adjacent, heavy
  // (late) query tiles first ----
  const int G = p.Hq / p.Hkv;
  int idx = blockIdx.x;
  const int g = idx % G;
  idx /= G;
  const int hkv = idx % p.Hkv;
  idx /= p.Hkv;
  const int b = idx % p.B;
  idx /= p.B;
  const int qt = p.n_qtiles - 1 - idx;
  const int hq = hkv * G + g;
  const int q0 = qt * kBM;
  const int offset = p.Tk - p.Tq;
  int n_kv;
  if (p.causal) {
    int last = q0 + kBM - 1 + offset;
    if (last > p.Tk - 1) last = p.Tk - 1;
    n_kv = last < 0 ? 0 : last / kBN + 1;
  } else {
    n_kv = (p.Tk + kBN - 1) / kBN;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
    }
    mbar_init(&pv_bar[0], 1);
    mbar_init(&pv_bar[1], 1);
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kColO = 256;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tmQ, q_full, 0, q0, hq, b);
      tma_load_4d(sQ + kHalfBytes, &tmQ, q_full, 64, q0, hq, b);
      int last_k = -1, last_v = -1;
      for (int j = 0; j < n_kv && !*abort_flag; ++j) {
        const int ks = j % kKS;
        const uint32_t ph = (j / kKS) & 1;
        if (!mbar_wait(&k_empty[ks], ph ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
        tma_load_4d(sK + ks * kTileBytes, &tmK, &k_full[ks], 0, j * kBN, hkv, b);
        tma_load_4d(sK + ks * kTileBytes + kHalfBytes, &tmK, &k_full[ks], 64, j * kBN, hkv, b);
        last_k = j;
        if (!mbar_wait(&v_empty[ks], ph ^ 1u, p.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[ks], kTileBytes);
        tma_load_4d(sV + ks * kTileBytes, &tmV, &v_full[ks], 0, j * kBN, hkv, b);
        tma_load_4d(sV + ks * kTileBytes + kHalfBytes, &tmV, &v_full[ks], 64, j * kBN, hkv, b);
        last_v = j;
      }
      // Drain: every issued TMA load has landed before teardown (on the normal
      // path the MMA warp has already consumed them all).
      mbar_wait(q_full, 0, p.status);
      for (int j = last_k; j >= 0 && j > last_k - kKS; --j) mbar_wait(&k_full[j % kKS], (j / kKS) & 1, p.status);
      for (int j = last_v; j >= 0 && j > last_v - kKS; --j) mbar_wait(&v_full[j % kKS], (j / kKS) & 1, p.status);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_bf16(kBM, kBN, false, false);
      constexpr uint32_t id_pv = make_idesc_bf16(kBM, kHeadDim, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int i) -> bool {
        const int vs = i % kKS;
        const uint32_t vph = (i / kKS) & 1;
        if (!mbar_wait(&v_full[vs], vph, p.status)) return false;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + vs * kTileBytes);
        const uint32_t p_tmem = tmem + (i & 1) * 128;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          umma_ts(tmem + kColO, p_tmem + k * 8, desc_mnmajor_sw128(v_addr + k * 2048, kHalfBytes), id_pv,
                  (i > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&pv_bar[i & 1]);
        tc_commit(&v_empty[vs]);
        if (i == n_kv - 1) tc_commit(o_full);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.status);
      if (ok) tc_fence_after();
      for (int j = 0; ok && j < n_kv; ++j) {
        const int ks = j % kKS;
        const uint32_t kph = (j / kKS) & 1;
        if (!mbar_wait(&k_full[ks], kph, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + ks * kTileBytes);
        const uint32_t d = tmem + (j & 1) * 128;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_ss(d, desc_kmajor_sw128(q_addr + off), desc_kmajor_sw128(k_addr + off), id_s, k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[j & 1]);
        tc_commit(&k_empty[ks]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
        if (*abort_flag) ok = false;
      }
      if (ok && n_kv > 0) ok = issue_pv(n_kv - 1);
      if (!ok) *abort_flag = 1;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------- softmax --
    const int r = (warp - 4) * 32 + lane;
    const int q = q0 + r;
    const int qlim = p.causal ? q + offset : p.Tk - 1;  // last visible key
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp - 4) * 32) << 16);
    float m_used = -INFINITY;
    float z = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int buf = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[buf], (j >> 1) & 1, p.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[128];
      tmem_ld32(lane_addr + buf * 128 + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld32(lane_addr + buf * 128 + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_ld32(lane_addr + buf * 128 + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
      tmem_ld32(lane_addr + buf * 128 + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
      tmem_wait_ld();
      const int kbase = j * kBN;
      if (kbase + kBN - 1 > qlim) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (kbase + c > qlim) s[c] = 0xFF800000u;  // -inf
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(s[c]));
      mx *= p.scale_log2;
      float alpha = 1.f;
      // The decision is warp-uniform (tcgen05.ld/st are warp-collective): when
      // any row of the warp needs a larger max, every row of the warp moves its
      // max up to max(m_used, mx), which is always valid for the online softmax.
      if (__any_sync(0xffffffffu, mx > m_used + kRescaleThreshold)) {
        const float m_new = fmaxf(m_used, mx);
        alpha = (m_new == m_used) ? 1.f : fast_exp2(m_used - m_new);  // 0 on the first tile
        if (j > 0) {
          // O holds P_0..P_{j-1} V: wait for the last PV, then rescale it.
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_bar[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t o[32];
            tmem_ld32(lane_addr + kColO + c4 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(lane_addr + kColO + c4 * 32, o);
          }
        }
        m_used = m_new;
      }
      const float msub = (m_used == -INFINITY) ? 0.f : m_used;
      float rowsum = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = fast_exp2(__uint_as_float(s[2 * c]) * p.scale_log2 - msub);
        const float p1 = fast_exp2(__uint_as_float(s[2 * c + 1]) * p.scale_log2 - msub);
        rowsum += p0 + p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      z = z * alpha + rowsum;
      tmem_st32(lane_addr + buf * 128 + 0, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
      tmem_st32(lane_addr + buf * 128 + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[buf]);
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: O / z and LSE ----
    if (__all_sync(0xffffffffu, ok && n_kv > 0 && mbar_wait(o_full, 0, p.status))) {
      tc_fence_after();
      const float inv = z > 0.f ? 1.f / z : 0.f;
      const bool row_ok = q < p.Tq;
      __nv_bfloat16* dst = p.o + (int64_t)b * p.o_sb + (int64_t)q * p.o_st + (int64_t)hq * p.o_sh;
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32(lane_addr + kColO + c4 * 32, o);
        tmem_wait_ld();
        if (row_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
            d4[v] = w;
          }
        }
      }
      if (row_ok && p.lse != nullptr) {
        p.lse[(int64_t)b * p.lse_sb + (int64_t)hq * p.lse_sh + q] =
            m_used * 0.69314718055994531f + __logf(z);
      }
    } else if (n_kv > 0) {
      *abort_flag = 1;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_attn_prefill(const __nv_bfloat16* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const __nv_bfloat16* k, const __nv_bfloat16* v, int64_t kv_sb, int64_t kv_sh,
                        int64_t kv_st, __nv_bfloat16* o, int64_t o_sb, int64_t o_st, int64_t o_sh, float* lse,
                        int64_t lse_sb, int64_t lse_sh, int B, int Hq, int Hkv, int Tq, int Tk, int head_dim,
                        int causal, float scale, cudaStream_t stream) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tq <= 0 || Tk <= 0)
    return set_error(kErrInvalidArgument, "attn_prefill: empty shape");
  if (head_dim != kHeadDim) return set_error(kErrUnsupported, "attn_prefill: head_dim must be 128");
  if (Hq % Hkv != 0) return set_error(kErrInvalidArgument, "attn_prefill: query heads must be a multiple of kv heads");
  if (causal && Tk < Tq) return set_error(kErrInvalidArgument, "attn_prefill: causal attention needs Tk >= Tq");
  if ((q_st % 8) || (q_sh % 8) || (q_sb % 8) || (kv_st % 8) || (kv_sh % 8) || (kv_sb % 8) || (o_st % 8) ||
      (o_sh % 8) || (o_sb % 8))
    return set_error(kErrInvalidArgument, "attn_prefill: strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return set_error(kErrInvalidArgument, "attn_prefill: tensors must be 16-byte aligned");

  CUtensorMap tmQ, tmK, tmV;
  const uint32_t box[4] = {64, 128, 1, 1};
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)Tq, (uint64_t)Hq, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)q_st * 2, (uint64_t)q_sh * 2, (uint64_t)q_sb * 2};
    int rc = make_tmap_bf16(&tmQ, q, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)Tk, (uint64_t)Hkv, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)kv_st * 2, (uint64_t)kv_sh * 2, (uint64_t)kv_sb * 2};
    int rc = make_tmap_bf16(&tmK, k, 4, dims, strides, box, true);
    if (rc) return rc;
    rc = make_tmap_bf16(&tmV, v, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  AttnParams p;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Tq = Tq;
  p.Tk = Tk;
  p.causal = causal;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_sb = o_sb;
  p.o_st = o_st;
  p.o_sh = o_sh;
  p.lse = lse;
  p.lse_sb = lse_sb;
  p.lse_sh = lse_sh;
  p.n_qtiles = (Tq + kBM - 1) / kBM;
  p.status = device_status_word();
  const int64_t grid = (int64_t)p.n_qtiles * B * Hq;
  if (grid > 0x7FFFFFFF) return set_error(kErrUnsupported, "attn_prefill: problem too large");
  int rc = check_cuda(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes),
                      "attn_prefill attr");
  if (rc) return rc;
  attn_prefill_kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, p);
  return check_cuda(cudaGetLastError(), "attn_prefill launch");
}

}  // namespace fmka
