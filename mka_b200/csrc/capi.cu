// C-ABI entry points of libfastmka_b200.so (declared in include/fastmka_b200.h):
// argument checking, the per-thread error channel, the per-device kernel status
// word, TMA tensor-map encoding, and the GEMM epilogue wiring for the Q/router
// and K/V projections.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/fastmka_b200.h"
#include "fmka_internal.h"

namespace fmka {

// Implemented in the kernel translation units.
size_t route_ema_blend_workspace_bytes(int B, int T, int D);
int launch_route_ema_blend(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, const __nv_bfloat16* l2,
                           int64_t l2_sb, int64_t l2_st, const float* logits,
                           const float* b2, const float* gate, int L, const __nv_bfloat16* l3, int64_t l3_sb,
                           int64_t l3_st, int T3, float beta, int B, int T, int D, __nv_bfloat16* h,
                           int64_t h_sb, int64_t h_st, float* lam, void* workspace, size_t workspace_bytes,
                           bool clear_flags, cudaStream_t stream, const float* ema_init = nullptr,
                           float* ema_final = nullptr, const struct KvOut* kv = nullptr);
int launch_route_ema_blend_kv(const __nv_bfloat16* y, int64_t y_sb, int64_t y_st, const float* logits, const float* b2,
                              const __nv_bfloat16* y3, int64_t y3_sb, int64_t y3_st, int T3, float beta, int B, int T, int Hkv, const float* bias, __nv_bfloat16* k_out,
                              __nv_bfloat16* v_out, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, int t_offset,
                              const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st,
                              float* lam, const float* ema_init, float* ema_final, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream);
size_t route_ema_blend_static_scratch_bytes();
int launch_route_ema_blend_static_scratch(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, const float* logits,
                                          const float* b2, const float* gate, int L, const __nv_bfloat16* l3,
                                          int64_t l3_sb, int64_t l3_st, int T3, float beta, int B, int T, int D,
                                          __nv_bfloat16* h, int64_t h_sb, int64_t h_st, float* lam,
                                          cudaStream_t stream);
int launch_attn_prefill(const __nv_bfloat16* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const __nv_bfloat16* k, const __nv_bfloat16* v, int64_t kv_sb, int64_t kv_sh,
                        int64_t kv_st, __nv_bfloat16* o, int64_t o_sb, int64_t o_st, int64_t o_sh, float* lse,
                        int64_t lse_sb, int64_t lse_sh, int B, int Hq, int Hkv, int Tq, int Tk, int head_dim,
                        int causal, float scale, cudaStream_t stream, const PeerPtrs* o_dst = nullptr,
                        int n_dst = 0, int rows_per_dst = 0);
int launch_peer_barrier(uint32_t* const* flags, int rank, int n, uint32_t epoch, cudaStream_t stream);
int launch_rmsnorm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w, float eps, __nv_bfloat16* y,
                   int64_t ldy, int rows, int D, cudaStream_t stream);
int launch_silu_mul(const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* out, int64_t n,
                    cudaStream_t stream);
int launch_block_mean(const __nv_bfloat16* x, int64_t x_sb, int64_t x_st, int B, int T, int D, int L,
                      __nv_bfloat16* q, int64_t ldq, cudaStream_t stream);
int launch_topr(const float* scores, int64_t lds, int M, int N, int R, float scale, int* idx, float* w,
                cudaStream_t stream);
int launch_recall_gather(const int* idx, const float* w, int R, const __nv_bfloat16* values, int64_t ldv, int nv,
                         int D, int B, int T, int L, __nv_bfloat16* out, int64_t o_sb, int64_t o_st,
                         cudaStream_t stream);
size_t attn_decode_workspace_bytes(int B, int Hq, int num_splits);
int attn_decode_plan(int B, int Hkv, int Tk, int requested, int* keys_per_split_out);
int launch_attn_decode(const __nv_bfloat16* q, int64_t q_sb, int64_t q_sh, const __nv_bfloat16* k,
                       const __nv_bfloat16* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, __nv_bfloat16* o,
                       int64_t o_sb, int64_t o_sh, float* lse, int64_t lse_sb, int B, int Hq, int Hkv, int Tk,
                       int head_dim, float scale, int num_splits, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream);

// ----------------------------------------------------------------- errors --
namespace {
thread_local int g_last_code = 0;
thread_local char g_last_msg[512] = {0};
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_code = code;
  std::snprintf(g_last_msg, sizeof(g_last_msg), "%s", msg.c_str());
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return kOk;
  return set_error(kErrCuda, std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------- per-device state --
namespace {
constexpr int kMaxDevices = 64;
__device__ uint32_t g_status_word;  // OR of FMKA_STATUS_* bits
uint32_t* g_status_ptr[kMaxDevices] = {nullptr};
int g_num_sms[kMaxDevices] = {0};
std::mutex g_dev_mu;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}
}  // namespace

uint32_t* device_status_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_status_ptr[dev] != nullptr) return g_status_ptr[dev];
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) == cudaSuccess) g_status_ptr[dev] = static_cast<uint32_t*>(p);
  }
  return g_status_ptr[dev];
}

int num_sms_current_device() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

// ------------------------------------------------------------ tensor maps --
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

namespace {
int make_tmap_typed(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return set_error(kErrCuda, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(kErrInvalidArgument, "TMA base address must be 16-byte aligned");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
    if (i > 0) {
      gstride[i - 1] = strides_bytes[i - 1];
      if (strides_bytes[i - 1] % 16 != 0)
        return set_error(kErrInvalidArgument, "TMA strides must be multiples of 16 bytes");
    }
  }
  CUresult r = g_encode(out, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kErrCuda, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return kOk;
}
}  // namespace

int make_tmap_bf16(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  return make_tmap_typed(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box, swizzle128);
}

int make_tmap_f32(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box) {
  return make_tmap_typed(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rank, dims, strides_bytes, box, false);
}

}  // namespace fmka

using namespace fmka;

namespace {
inline cudaStream_t as_stream(fmka_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// The projection epilogues read bias, RoPE rows and router rows as float4.
int check_epilogue_inputs(const float* bias, const float* cs, const float* sn, int64_t rope_sb, int64_t rope_st,
                          const char* who) {
  if (bias != nullptr && !al16(bias)) return set_error(kErrInvalidArgument, std::string(who) + ": bias must be 16-byte aligned");
  if (cs != nullptr && (!al16(cs) || !al16(sn) || (rope_sb % 4) || (rope_st % 4)))
    return set_error(kErrInvalidArgument, std::string(who) + ": RoPE tables must be 16-byte aligned with strides % 4 == 0");
  return kOk;
}
inline const __nv_bfloat16* bf(const void* p) { return static_cast<const __nv_bfloat16*>(p); }
inline __nv_bfloat16* bfw(void* p) { return static_cast<__nv_bfloat16*>(p); }

GemmSeg empty_seg() {
  GemmSeg s;
  std::memset(&s, 0, sizeof(s));
  return s;
}
}  // namespace

extern "C" {

const char* fmka_version(void) { return "fastmka_b200 0.1.0 (sm_100a)"; }

int fmka_get_last_error(char* buf, int buflen) {
  if (buf != nullptr && buflen > 0) std::snprintf(buf, (size_t)buflen, "%s", g_last_msg);
  return g_last_code;
}

int fmka_device_status(uint32_t* status, int clear, fmka_stream_t stream) {
  uint32_t* dev = device_status_word();
  if (dev == nullptr) return set_error(kErrDevice, "device status word unavailable");
  uint32_t host = 0;
  int rc = check_cuda(cudaMemcpyAsync(&host, dev, sizeof(host), cudaMemcpyDeviceToHost, as_stream(stream)),
                      "status read");
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(as_stream(stream)), "status sync");
  if (rc) return rc;
  if (clear) {
    rc = check_cuda(cudaMemsetAsync(dev, 0, sizeof(uint32_t), as_stream(stream)), "status clear");
    if (rc) return rc;
  }
  if (status) *status = host;
  return kOk;
}

int fmka_num_sms(void) { return num_sms_current_device(); }

int fmka_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, const float* bias, void* c, int64_t ldc,
                   int M, int N, int K, fmka_stream_t stream) {
  if (a == nullptr || w == nullptr || c == nullptr) return set_error(kErrInvalidArgument, "gemm: null pointer");
  if (bias != nullptr && !al16(bias)) return set_error(kErrInvalidArgument, "gemm: bias must be 16-byte aligned");
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_split = N;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegRowMajor;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = N;
  p.seg[0].out = bfw(c);
  p.seg[0].ld = ldc;
  p.seg[0].bias = bias;
  p.seg[1] = empty_seg();
  p.status = device_status_word();
  return launch_gemm(bf(a), lda, bf(w), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_gemm_bf16_f32out(const void* a, int64_t lda, const void* w, int64_t ldw, float* c, int64_t ldc, int M,
                          int N, int K, fmka_stream_t stream) {
  if (a == nullptr || w == nullptr || c == nullptr) return set_error(kErrInvalidArgument, "gemm: null pointer");
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_split = N;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegRowMajorF32;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = N;
  p.seg[0].out_f32 = c;
  p.seg[0].ld = ldc;
  p.seg[1] = empty_seg();
  p.status = device_status_word();
  return launch_gemm(bf(a), lda, bf(w), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_gemm_bf16_kblocked(const void* a, int a_kblk, int64_t a_blk_stride, int64_t lda, const void* w, int64_t ldw,
                            const float* bias, void* c, int64_t ldc, int M, int N, int K, fmka_stream_t stream) {
  if (a == nullptr || w == nullptr || c == nullptr) return set_error(kErrInvalidArgument, "gemm: null pointer");
  if (a_kblk <= 0) return set_error(kErrInvalidArgument, "gemm: a_kblk must be positive");
  if (bias != nullptr && !al16(bias)) return set_error(kErrInvalidArgument, "gemm: bias must be 16-byte aligned");
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_kblk = a_kblk;
  p.a_blk_stride = a_blk_stride;
  p.n_split = N;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegRowMajor;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = N;
  p.seg[0].out = bfw(c);
  p.seg[0].ld = ldc;
  p.seg[0].bias = bias;
  p.seg[1] = empty_seg();
  p.status = device_status_word();
  return launch_gemm(bf(a), lda, bf(w), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_gemm_bf16_swiglu(const void* a, int64_t lda, const void* w_gu, int64_t ldw, const float* bias_gu, void* c,
                          int64_t ldc, int M, int I, int K, fmka_stream_t stream) {
  if (a == nullptr || w_gu == nullptr || c == nullptr) return set_error(kErrInvalidArgument, "gemm_swiglu: null pointer");
  if (I <= 0 || I % 128 != 0)
    return set_error(kErrInvalidArgument, "gemm_swiglu: the channel count must be a positive multiple of 128");
  if (bias_gu != nullptr && !al16(bias_gu))
    return set_error(kErrInvalidArgument, "gemm_swiglu: bias must be 16-byte aligned");
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = 2 * I;
  p.K = K;
  p.n_split = 2 * I;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegSwiGLU;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = 2 * I;
  p.seg[0].out = bfw(c);
  p.seg[0].ld = ldc;
  p.seg[0].bias = bias_gu;
  p.seg[1] = empty_seg();
  p.status = device_status_word();
  return launch_gemm(bf(a), lda, bf(w_gu), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_qr_proj(const void* x, int64_t ldx, const void* w_qr, int64_t ldw, const float* bias_qr, int B, int T,
                 int D, int Hq, int R, void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, int t_offset,
                 const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st, const float* w2,
                 int L, int act, float* logits, fmka_stream_t stream) {
  if (x == nullptr || w_qr == nullptr || q == nullptr) return set_error(kErrInvalidArgument, "qr_proj: null pointer");
  if (B <= 0 || T <= 0 || D <= 0 || Hq <= 0 || R < 0) return set_error(kErrInvalidArgument, "qr_proj: bad shape");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return set_error(kErrInvalidArgument, "qr_proj: pass both rope cos and sin or neither");
  if (act != 0 && act != 1) return set_error(kErrInvalidArgument, "qr_proj: act must be 0 (SiLU) or 1 (GELU)");
  if ((q_sb % 8) || (q_sh % 8) || (q_st % 8)) return set_error(kErrInvalidArgument, "qr_proj: q strides % 8");
  if (int rc = check_epilogue_inputs(bias_qr, rope_cos, rope_sin, rope_sb, rope_st, "qr_proj")) return rc;
  if (w2 != nullptr && !al16(w2)) return set_error(kErrInvalidArgument, "qr_proj: w2 must be 16-byte aligned");
  const int Nq = Hq * 128;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = B * T;
  p.N = Nq + R;
  p.K = D;
  p.n_split = Nq;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegHeads;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = Nq;
  p.seg[0].out = bfw(q);
  p.seg[0].bias = bias_qr;
  p.seg[0].T = T;
  p.seg[0].head_dim = 128;
  p.seg[0].s_b = q_sb;
  p.seg[0].s_h = q_sh;
  p.seg[0].s_t = q_st;
  p.seg[0].t_offset = t_offset;
  p.seg[0].rope_cos = rope_cos;
  p.seg[0].rope_sin = rope_sin;
  p.seg[0].rope_sb = rope_sb;
  p.seg[0].rope_st = rope_st;
  p.seg[1] = empty_seg();
  if (R > 0) {
    if (w2 == nullptr || logits == nullptr || L < 1 || L > 4)
      return set_error(kErrInvalidArgument, "qr_proj: router needs w2, logits and 1..4 levels");
    p.seg[1].kind = kSegRouter;
    p.seg[1].n_begin = Nq;
    p.seg[1].n_end = Nq + R;
    p.seg[1].bias = bias_qr ? bias_qr + Nq : nullptr;
    p.seg[1].w2 = w2;
    p.seg[1].L = L;
    p.seg[1].act = act;
    p.seg[1].logits = logits;
  }
  p.status = device_status_word();
  return launch_gemm(bf(x), ldx, bf(w_qr), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_kv_proj(const void* h, int64_t ldh, const void* w_kv, int64_t ldw, const float* bias_kv, int B, int T,
                 int D, int Hkv, void* k, void* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, int t_offset,
                 const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st,
                 fmka_stream_t stream) {
  if (h == nullptr || w_kv == nullptr || k == nullptr || v == nullptr)
    return set_error(kErrInvalidArgument, "kv_proj: null pointer");
  if (B <= 0 || T <= 0 || D <= 0 || Hkv <= 0) return set_error(kErrInvalidArgument, "kv_proj: bad shape");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return set_error(kErrInvalidArgument, "kv_proj: pass both rope cos and sin or neither");
  if ((kv_sb % 8) || (kv_sh % 8) || (kv_st % 8)) return set_error(kErrInvalidArgument, "kv_proj: kv strides % 8");
  if (int rc = check_epilogue_inputs(bias_kv, rope_cos, rope_sin, rope_sb, rope_st, "kv_proj")) return rc;
  const int Nk = Hkv * 128;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = B * T;
  p.N = 2 * Nk;
  p.K = D;
  p.n_split = Nk;
  for (int s = 0; s < 2; ++s) {
    p.seg[s] = empty_seg();
    p.seg[s].kind = kSegHeads;
    p.seg[s].n_begin = s * Nk;
    p.seg[s].n_end = (s + 1) * Nk;
    p.seg[s].out = bfw(s == 0 ? k : v);
    p.seg[s].bias = bias_kv ? bias_kv + s * Nk : nullptr;
    p.seg[s].T = T;
    p.seg[s].head_dim = 128;
    p.seg[s].s_b = kv_sb;
    p.seg[s].s_h = kv_sh;
    p.seg[s].s_t = kv_st;
    p.seg[s].t_offset = t_offset;
  }
  p.seg[0].rope_cos = rope_cos;
  p.seg[0].rope_sin = rope_sin;
  p.seg[0].rope_sb = rope_sb;
  p.seg[0].rope_st = rope_st;
  p.status = device_status_word();
  return launch_gemm(bf(h), ldh, bf(w_kv), ldw, p, num_sms_current_device(), as_stream(stream));
}

size_t fmka_route_ema_blend_workspace_size(int B, int T, int D) {
  if (B <= 0 || T <= 0 || D <= 0) return 0;
  return route_ema_blend_workspace_bytes(B, T, D);
}

int fmka_route_ema_blend(const void* x, int64_t x_sb, int64_t x_st, const float* logits, const float* b2,
                         const float* gate, int L, const void* l3, int64_t l3_sb, int64_t l3_st, int T3, float beta,
                         int B, int T, int D, void* h, int64_t h_sb, int64_t h_st, float* lam, void* workspace,
                         size_t workspace_bytes, fmka_stream_t stream) {
  if (x == nullptr || h == nullptr) return set_error(kErrInvalidArgument, "route_ema_blend: null pointer");
  if (!std::isfinite(beta)) return set_error(kErrInvalidArgument, "route_ema_blend: beta must be finite");
  return launch_route_ema_blend(bf(x), x_sb, x_st, nullptr, 0, 0, logits, b2, gate, L, bf(l3), l3_sb, l3_st, T3,
                                beta, B, T, D, bfw(h), h_sb, h_st, lam, workspace, workspace_bytes, true,
                                as_stream(stream));
}

int fmka_route_ema_blend_noalloc(const void* x, int64_t x_sb, int64_t x_st, const float* logits, const float* b2,
                                 const float* gate, int L, const void* l3, int64_t l3_sb, int64_t l3_st, int T3,
                                 float beta, int B, int T, int D, void* h, int64_t h_sb, int64_t h_st, float* lam,
                                 fmka_stream_t stream) {
  if (x == nullptr || h == nullptr) return set_error(kErrInvalidArgument, "route_ema_blend_noalloc: null pointer");
  if (!std::isfinite(beta)) return set_error(kErrInvalidArgument, "route_ema_blend_noalloc: beta must be finite");
  return launch_route_ema_blend_static_scratch(bf(x), x_sb, x_st, logits, b2, gate, L, bf(l3), l3_sb, l3_st, T3, beta,
                                               B, T, D, bfw(h), h_sb, h_st, lam, as_stream(stream));
}

size_t fmka_route_ema_blend_noalloc_scratch_bytes(void) { return route_ema_blend_static_scratch_bytes(); }

int fmka_route_ema_blend_state(const void* x, int64_t x_sb, int64_t x_st, const float* logits, const float* b2,
                               const float* gate, int L, const void* l3, int64_t l3_sb, int64_t l3_st, int T3,
                               float beta, int B, int T, int D, void* h, int64_t h_sb, int64_t h_st, float* lam,
                               const float* ema_init, float* ema_final, void* workspace, size_t workspace_bytes,
                               fmka_stream_t stream) {
  if (x == nullptr || h == nullptr) return set_error(kErrInvalidArgument, "route_ema_blend_state: null pointer");
  if (!std::isfinite(beta)) return set_error(kErrInvalidArgument, "route_ema_blend_state: beta must be finite");
  if (ema_init != nullptr && ema_init == ema_final)
    return set_error(kErrInvalidArgument, "route_ema_blend_state: ema_init and ema_final must not alias");
  return launch_route_ema_blend(bf(x), x_sb, x_st, nullptr, 0, 0, logits, b2, gate, L, bf(l3), l3_sb, l3_st, T3,
                                beta, B, T, D, bfw(h), h_sb, h_st, lam, workspace, workspace_bytes, true,
                                as_stream(stream), ema_init, ema_final);
}

size_t fmka_route_ema_blend_kv_workspace_size(int B, int T, int Hkv) {
  if (B <= 0 || T <= 0 || Hkv <= 0) return 0;
  return route_ema_blend_workspace_bytes(B, T, 2 * Hkv * 128);
}

int fmka_route_ema_blend_kv(const void* y, int64_t y_sb, int64_t y_st, const float* logits, const float* b2,
                            const void* y3, int64_t y3_sb, int64_t y3_st, int T3, float beta, int B, int T, int Hkv, const float* bias, void* k_out, void* v_out,
                            int64_t kv_sb, int64_t kv_sh, int64_t kv_st, int t_offset, const float* rope_cos,
                            const float* rope_sin, int64_t rope_sb, int64_t rope_st, float* lam,
                            const float* ema_init, float* ema_final, void* workspace, size_t workspace_bytes,
                            fmka_stream_t stream) {
  if (y == nullptr) return set_error(kErrInvalidArgument, "route_ema_blend_kv: null pointer");
  if (!std::isfinite(beta)) return set_error(kErrInvalidArgument, "route_ema_blend_kv: beta must be finite");
  if (ema_init != nullptr && ema_init == ema_final)
    return set_error(kErrInvalidArgument, "route_ema_blend_kv: ema_init and ema_final must not alias");
  if (y3 != nullptr && T3 < 1) return set_error(kErrInvalidArgument, "route_ema_blend_kv: y3 needs T3 >= 1");
  return launch_route_ema_blend_kv(bf(y), y_sb, y_st, logits, b2, bf(y3), y3_sb, y3_st, T3, beta, B, T, Hkv, bias, bfw(k_out), bfw(v_out),
                                   kv_sb, kv_sh, kv_st, t_offset, rope_cos, rope_sin, rope_sb, rope_st, lam,
                                   ema_init, ema_final, workspace, workspace_bytes, as_stream(stream));
}

int fmka_route_blend(const void* l1, int64_t l1_sb, int64_t l1_st, const void* l2, int64_t l2_sb, int64_t l2_st,
                     const void* l3, int64_t l3_sb, int64_t l3_st, int T3, const float* gate, int L, int B, int T,
                     int D, void* h, int64_t h_sb, int64_t h_st, fmka_stream_t stream) {
  if (l1 == nullptr || l2 == nullptr || gate == nullptr || h == nullptr)
    return set_error(kErrInvalidArgument, "route_blend: null pointer");
  return launch_route_ema_blend(bf(l1), l1_sb, l1_st, bf(l2), l2_sb, l2_st, nullptr, nullptr, gate, L, bf(l3), l3_sb,
                                l3_st, T3, 0.f, B, T, D, bfw(h), h_sb, h_st, nullptr, nullptr, 0, false,
                                as_stream(stream));
}

int fmka_attn_fwd_prefill(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k, const void* v,
                          int64_t kv_sb, int64_t kv_sh, int64_t kv_st, void* o, int64_t o_sb, int64_t o_st,
                          int64_t o_sh, float* lse, int64_t lse_sb, int64_t lse_sh, int B, int Hq, int Hkv, int Tq,
                          int Tk, int head_dim, int causal, float scale, fmka_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return set_error(kErrInvalidArgument, "attn_prefill: null pointer");
  return launch_attn_prefill(bf(q), q_sb, q_sh, q_st, bf(k), bf(v), kv_sb, kv_sh, kv_st, bfw(o), o_sb, o_st, o_sh,
                             lse, lse_sb, lse_sh, B, Hq, Hkv, Tq, Tk, head_dim, causal, scale, as_stream(stream));
}

int fmka_rmsnorm_bf16(const void* x, int64_t ldx, const void* w, float eps, void* y, int64_t ldy, int rows, int D,
                      fmka_stream_t stream) {
  if (x == nullptr || w == nullptr || y == nullptr) return set_error(kErrInvalidArgument, "rmsnorm: null pointer");
  if (!std::isfinite(eps) || eps < 0.f) return set_error(kErrInvalidArgument, "rmsnorm: eps must be finite and >= 0");
  return launch_rmsnorm(bf(x), ldx, bf(w), eps, bfw(y), ldy, rows, D, as_stream(stream));
}

int fmka_silu_mul_bf16(const void* g, const void* u, void* out, int64_t n, fmka_stream_t stream) {
  if (g == nullptr || u == nullptr || out == nullptr) return set_error(kErrInvalidArgument, "silu_mul: null pointer");
  return launch_silu_mul(bf(g), bf(u), bfw(out), n, as_stream(stream));
}

int fmka_l3_block_mean_bf16(const void* x, int64_t x_sb, int64_t x_st, int B, int T, int D, int block_len,
                            void* q, int64_t ldq, fmka_stream_t stream) {
  if (x == nullptr || q == nullptr) return set_error(kErrInvalidArgument, "block_mean: null pointer");
  return launch_block_mean(bf(x), x_sb, x_st, B, T, D, block_len, bfw(q), ldq, as_stream(stream));
}

int fmka_l3_topr_f32(const float* scores, int64_t lds, int M, int N, int R, float scale, int32_t* idx, float* w,
                     fmka_stream_t stream) {
  if (scores == nullptr || idx == nullptr || w == nullptr) return set_error(kErrInvalidArgument, "topr: null pointer");
  if (!std::isfinite(scale)) return set_error(kErrInvalidArgument, "topr: scale must be finite");
  return launch_topr(scores, lds, M, N, R, scale, idx, w, as_stream(stream));
}

int fmka_l3_recall_gather_bf16(const int32_t* idx, const float* w, int R, const void* values, int64_t ldv, int n_chunks,
                               int D, int B, int T, int block_len, void* out, int64_t o_sb, int64_t o_st,
                               fmka_stream_t stream) {
  if (idx == nullptr || w == nullptr || values == nullptr || out == nullptr)
    return set_error(kErrInvalidArgument, "recall_gather: null pointer");
  return launch_recall_gather(idx, w, R, bf(values), ldv, n_chunks, D, B, T, block_len, bfw(out), o_sb, o_st,
                              as_stream(stream));
}

int fmka_attn_fwd_prefill_scatter(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                                  const void* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, void* const* o_dst,
                                  int n_dst, int rows_per_dst, int64_t o_sb, int64_t o_st, int64_t o_sh, int B,
                                  int Hq, int Hkv, int Tq, int Tk, int head_dim, int causal, float scale,
                                  fmka_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o_dst == nullptr)
    return set_error(kErrInvalidArgument, "attn_prefill_scatter: null pointer");
  if (n_dst < 1 || n_dst > kMaxPeers)
    return set_error(kErrInvalidArgument, "attn_prefill_scatter: 1 to 8 destinations");
  PeerPtrs d;
  for (int j = 0; j < kMaxPeers; ++j) d.p[j] = j < n_dst ? static_cast<__nv_bfloat16*>(o_dst[j]) : nullptr;
  return launch_attn_prefill(bf(q), q_sb, q_sh, q_st, bf(k), bf(v), kv_sb, kv_sh, kv_st, d.p[0], o_sb, o_st, o_sh,
                             nullptr, 0, 0, B, Hq, Hkv, Tq, Tk, head_dim, causal, scale, as_stream(stream), &d, n_dst,
                             rows_per_dst);
}

int fmka_gemm_bf16_kblocked_scatter(const void* a, int a_kblk, int64_t a_blk_stride, int64_t lda, const void* w,
                                    int64_t ldw, const float* bias, void* const* c_dst, int n_dst, int64_t c_row0,
                                    int64_t ldc, int M, int N, int K, fmka_stream_t stream) {
  if (a == nullptr || w == nullptr || c_dst == nullptr) return set_error(kErrInvalidArgument, "gemm: null pointer");
  if (a_kblk <= 0) return set_error(kErrInvalidArgument, "gemm: a_kblk must be positive");
  if (n_dst < 1 || n_dst > kMaxPeers) return set_error(kErrInvalidArgument, "gemm: 1 to 8 scatter destinations");
  if (bias != nullptr && !al16(bias)) return set_error(kErrInvalidArgument, "gemm: bias must be 16-byte aligned");
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_kblk = a_kblk;
  p.a_blk_stride = a_blk_stride;
  p.n_split = N;
  p.seg[0] = empty_seg();
  p.seg[0].kind = kSegRowMajor;
  p.seg[0].n_begin = 0;
  p.seg[0].n_end = N;
  p.seg[0].bias = bias;
  p.seg[1] = empty_seg();
  p.status = device_status_word();
  p.n_dst = n_dst;
  p.dst_row0 = c_row0;
  p.dst_ld = ldc;
  for (int j = 0; j < kMaxPeers; ++j) p.dst.p[j] = j < n_dst ? static_cast<__nv_bfloat16*>(c_dst[j]) : nullptr;
  return launch_gemm(bf(a), lda, bf(w), ldw, p, num_sms_current_device(), as_stream(stream));
}

int fmka_peer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return set_error(kErrInvalidArgument, "peer_alloc: null pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, bytes), "peer_alloc");
  if (rc) return rc;
  rc = check_cuda(cudaMemset(p, 0, bytes), "peer_alloc zero");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return kOk;
}

int fmka_peer_free(void* ptr) {
  if (ptr == nullptr) return kOk;
  return check_cuda(cudaFree(ptr), "peer_free");
}

static_assert(sizeof(cudaIpcMemHandle_t) == FMKA_PEER_HANDLE_BYTES, "IPC handle size");

int fmka_peer_export(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return set_error(kErrInvalidArgument, "peer_export: null pointer");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "peer_export");
  if (rc) return rc;
  std::memcpy(handle, &h, sizeof(h));
  return kOk;
}

int fmka_peer_import(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return set_error(kErrInvalidArgument, "peer_import: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer_import");
}

int fmka_peer_close(void* ptr) {
  if (ptr == nullptr) return kOk;
  return check_cuda(cudaIpcCloseMemHandle(ptr), "peer_close");
}

int fmka_peer_barrier(uint32_t* const* flags, int rank, int n, uint32_t epoch, fmka_stream_t stream) {
  if (flags == nullptr) return set_error(kErrInvalidArgument, "peer_barrier: null pointer");
  return launch_peer_barrier(flags, rank, n, epoch, as_stream(stream));
}

int fmka_attn_decode_num_splits(int B, int Hkv, int Tk) {
  if (B <= 0 || Hkv <= 0 || Tk <= 0) return 1;
  return attn_decode_plan(B, Hkv, Tk, 0, nullptr);
}

size_t fmka_attn_decode_workspace_size(int B, int Hq, int Hkv, int Tk, int num_splits) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Tk <= 0) return 0;
  const int s = attn_decode_plan(B, Hkv, Tk, num_splits, nullptr);
  return attn_decode_workspace_bytes(B, Hq, s);
}

int fmka_attn_decode_splitkv(const void* q, int64_t q_sb, int64_t q_sh, const void* k, const void* v, int64_t kv_sb,
                             int64_t kv_sh, int64_t kv_st, void* o, int64_t o_sb, int64_t o_sh, float* lse,
                             int64_t lse_sb, int B, int Hq, int Hkv, int Tk, int head_dim, float scale,
                             int num_splits, void* workspace, size_t workspace_bytes, fmka_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return set_error(kErrInvalidArgument, "attn_decode: null pointer");
  return launch_attn_decode(bf(q), q_sb, q_sh, bf(k), bf(v), kv_sb, kv_sh, kv_st, bfw(o), o_sb, o_sh, lse, lse_sb,
                            B, Hq, Hkv, Tk, head_dim, scale, num_splits, workspace, workspace_bytes,
                            as_stream(stream));
}

}  // extern "C"
