// Internal declarations shared by the FastMKA CUDA translation units: launch
// parameter structs, kernel launchers and the per-thread error channel that the
// C-ABI entry points report through.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace fmka {

// ----------------------------------------------------------------- errors --
// Status codes returned by every C-ABI entry point (0 = success).
enum Status : int {
  kOk = 0,
  kErrInvalidArgument = 1,
  kErrUnsupported = 2,
  kErrCuda = 3,
  kErrWorkspace = 4,
  kErrDevice = 5,
};

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
// Checks a CUDA runtime result; on failure records it and returns kErrCuda.
int check_cuda(cudaError_t e, const char* what);

// ------------------------------------------------------------- tensor maps --
// Encodes a bf16 tiled tensor map (rank 2 to 5), with or without 128-byte swizzle.
// dims/strides are innermost first; strides are in bytes for dims 1..rank-1.
int make_tmap_bf16(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);
// The same for fp32 elements, without swizzle.
int make_tmap_f32(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box);

// ------------------------------------------------------------ peer memory --
// Most ranks (GPUs of one box) that exchange data through peer mappings.
constexpr int kMaxPeers = 8;

// Pointers into the same buffer as mapped in each rank (index = rank in group).
struct PeerPtrs {
  __nv_bfloat16* p[kMaxPeers];
};

// ------------------------------------------------------------------- GEMM --
enum SegKind : int { kSegRowMajor = 0, kSegHeads = 1, kSegRouter = 2, kSegSwiGLU = 3, kSegRowMajorF32 = 4 };

struct GemmSeg {
  int kind;
  int n_begin;           // first global column of this segment
  int n_end;             // one past the last column of this segment
  __nv_bfloat16* out;    // row-major: [M, ld]; heads: [B, H, Tcap, Dh] through strides
  int64_t ld;            // row-major row stride (elements)
  const float* bias;     // indexed by (n - n_begin); may be null
  int T;                 // tokens per batch row (rows m = b*T + t)
  int head_dim;          // 128
  int64_t s_b, s_h, s_t; // element strides of the head-split output
  int t_offset;          // first token slot written in the head-split output
  const float* rope_cos; // [*, T, head_dim] fp32 or null (no RoPE)
  const float* rope_sin;
  int64_t rope_sb, rope_st;
  const float* w2;       // router second layer [L, R] fp32
  int L;
  int act;               // 0 = SiLU, 1 = GELU (erf)
  float* logits;         // [M, L] fp32, accumulated
  float* out_f32;        // kSegRowMajorF32: [M, ld] fp32 output (row stride ld)
  // SwiGLU: columns come in blocks of 256, gate rows then up rows of the same
  // 128 output channels; out [M, ld] receives silu(gate) * up per channel.
};

struct GemmParams {
  int M, N, K;
  int a_kblk;            // > 0: A is stored as K / a_kblk blocks of [M, a_kblk]
  int64_t a_blk_stride;  // element distance between those blocks
  int n_split;  // columns < n_split use seg[0], the rest seg[1]
  GemmSeg seg[2];
  uint32_t* status;
  // Scatter epilogue (n_dst > 0, replaces the segments): bias seg[0].bias,
  // output row m written to row dst_row0 + m of every dst.p[0 .. n_dst-1]
  // (row stride dst_ld), each a local or a peer-mapped [*, N] bf16 buffer.
  int n_dst;
  int64_t dst_row0;
  int64_t dst_ld;
  PeerPtrs dst;
  // Tile order (set by launch_gemm): bands of raster_group row blocks with the
  // row block running fastest inside a band; 1 is plain row-major order.
  int raster_group;
};

// Row block mb and column block nb of persistent-GEMM tile `tile` (see
// GemmParams::raster_group); a bijection of [0, num_m * num_n) onto the grid.
__host__ __device__ __forceinline__ void gemm_tile_coords(int tile, int num_m, int num_n, int group, int& mb,
                                                          int& nb) {
  const int band_tiles = group * num_n;
  const int band = tile / band_tiles;
  const int first = band * group;
  const int rows = group < num_m - first ? group : num_m - first;
  const int r = tile - band * band_tiles;
  mb = first + r % rows;
  nb = r / rows;
}

// C = A[M,K] * B[N,K]^T with the segment epilogues. A and B are row-major bf16
// with row strides lda / ldb (elements).
int launch_gemm(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb, const GemmParams& p,
                int num_sms, cudaStream_t stream);

// Device status word used by kernels to report bounded-wait timeouts; one per
// device, allocated lazily.
uint32_t* device_status_word();
int num_sms_current_device();

}  // namespace fmka
