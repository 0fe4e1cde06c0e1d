// Internal layout contract shared by the kernels and the C ABI: packed-weight offsets, workspace
// regions and the attention-oriented strided views of z / mask / out.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace triattn {

constexpr int C_IN = 128;
constexpr int HEADS = 4;
constexpr int C_HEAD = 32;
constexpr int HC = HEADS * C_HEAD;  // 128
constexpr int NPROJ = 4 * HC;       // 512 = q|k|v|g
constexpr float LN_EPS = 1e-5f;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float QSCALE_L2 = 0.17677669529663687f * 1.4426950408889634f;  // C^-1/2 * log2(e)
constexpr int TILE = 128;  // query / key / pair tile of the tensor-core path

constexpr int DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2;

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
__host__ __device__ constexpr int round_tile(int n) { return (n + TILE - 1) / TILE * TILE; }

// ---- packed weights ---------------------------------------------------------------------------
// fp32 section (floats): ln_w[128] ln_b[128] g_b[128] w_b[4][128] w_qkvg[512][128] w_o[128][128]
// 16-bit section: W_qkvg operand image (K-major, 512 rows x 128 k), W_o operand image (128 x 128).
struct PackedLayout {
  static constexpr size_t ln_w = 0;
  static constexpr size_t ln_b = ln_w + C_IN * 4;
  static constexpr size_t g_b = ln_b + C_IN * 4;
  static constexpr size_t w_b = g_b + HC * 4;
  static constexpr size_t w_qkvg = w_b + HEADS * C_IN * 4;
  static constexpr size_t w_o = w_qkvg + NPROJ * C_IN * 4;
  static constexpr size_t f32_end = w_o + C_IN * HC * 4;
  static constexpr size_t img_qkvg = align_up(f32_end, 1024);
  static constexpr size_t img_o = img_qkvg + NPROJ * C_IN * 2;
  static constexpr size_t end16 = img_o + C_IN * HC * 2;
  static constexpr size_t bytes(int dtype) { return dtype == DT_F32 ? align_up(f32_end, 256) : align_up(end16, 256); }
};

// ---- workspace ---------------------------------------------------------------------------------
// The tri-bias region comes first, at offset 0, so it sits at the same place whatever row count a
// call is made with: row chunks of different sizes (and the ranks of a row-sharded layer) fill and
// read one shared bias.  Per-row regions follow, laid out for R = row_end - row_begin.
// 16-bit path (NT = Np / 128 tiles, Np = N rounded up to 128):
//   bias     : fp16, log2 domain, 128 x 128 blocks [qt][b][h][kt], each block stored [k/8][q][8]
//              (a query's 8 consecutive keys are 16 contiguous bytes; 2 KB between key groups)
//   q_img    : [B][R][H][NT] tiles of 8 KB, K-major 128 x 32 image, q pre-scaled by C^-1/2 log2(e)
//   k_img    : [B][R][H][NT] tiles of 8 KB, K-major 128 x 32 image
//   v_img    : [B][R][H][NT] tiles of 8 KB, fp16, MN-major image: byte(key, ch) =
//              (ch/8)*2048 + (key/8)*128 + (key%8)*16 + (ch%8)*2
//   g        : [B][R][N][128] 16-bit
//   core_img : [B][R][NT] tiles of 32 KB (128 positions x 128 channels, K-major image)
//   mb       : [B][R][Np] fp32, log2-domain mask bias; padded keys -1e30
//   ts       : [B][R][NTs] uint8 key-tile class: 0 all keys valid, 1 all masked (skip), 2 mixed;
//              NTs = NT rounded up to 4 (one aligned 32-bit word per 4 tiles)
// fp32 path:
//   bias     : [N][B][H][Np] fp32 tri bias (natural units)
//   q (pre-scaled by C^-1/2), k, v, g, core : [B][R][N][128] fp32;  mb : [B][R][Np] = inf * (mask - 1)
struct Workspace {
  int B, N, R, dtype, Np, NT, NTs;
  size_t off_q, off_k, off_v, off_g, off_core, off_bias, off_mb, off_ts, total;

  __host__ __device__ static Workspace make(int B, int N, int R, int dtype) {
    Workspace w{};
    w.B = B; w.N = N; w.R = R; w.dtype = dtype;
    w.Np = round_tile(N);
    w.NT = w.Np / TILE;
    w.NTs = (w.NT + 3) / 4 * 4;
    const size_t A = 256;
    size_t o = 0;
    w.off_bias = o;
    o = align_up(o + (dtype == DT_F32 ? (size_t)N * B * HEADS * w.Np * 4 : (size_t)w.Np * B * HEADS * w.Np * 2), A);
    if (dtype == DT_F32) {
      const size_t plane = (size_t)B * R * N * C_IN * 4;
      w.off_q = o; o = align_up(o + plane, A);
      w.off_k = o; o = align_up(o + plane, A);
      w.off_v = o; o = align_up(o + plane, A);
      w.off_g = o; o = align_up(o + plane, A);
      w.off_core = o; o = align_up(o + plane, A);
    } else {
      const size_t head_tiles = (size_t)B * R * HEADS * w.NT * 8192;
      w.off_q = o; o = align_up(o + head_tiles, A);
      w.off_k = o; o = align_up(o + head_tiles, A);
      w.off_v = o; o = align_up(o + head_tiles, A);
      w.off_g = o; o = align_up(o + (size_t)B * R * N * C_IN * 2, A);
      w.off_core = o; o = align_up(o + (size_t)B * R * w.NT * 32768, A);
    }
    w.off_mb = o; o = align_up(o + (size_t)B * R * w.Np * 4, A);
    w.off_ts = o; o = align_up(o + (size_t)B * R * w.NTs, A);
    w.total = o;
    return w;
  }
};

// ---- triangle multiplication (outgoing / incoming edges) -----------------------------------------
// packed weights: fp32 section: in_w, in_b, out_w, out_b [128 each]; W1 = p_in | g_in | g_out
// [640][128]; p_out [128][128].  16-bit section (16-bit modes): W1 and p_out in the layer's type,
// row-major, and as K-major no-swizzle UMMA operand images (img_off) for the fused projection and
// tail kernels: img_pg = 640 rows p_in[0:128] | g_in[0:128] | p_in[128:256] | g_in[128:256] | g_out
// (the a half, the b half, then the output gate), img_po = p_out (128 x 128).
constexpr int TM_D = 128;
constexpr int TM_W1 = 5 * TM_D;  // 640 = p_in (256) | g_in (256) | g_out (128)
struct TrimulPacked {
  static constexpr size_t in_w = 0, in_b = 512, out_w = 1024, out_b = 1536;
  static constexpr size_t w1 = 2048;
  static constexpr size_t p_out = w1 + (size_t)TM_W1 * TM_D * 4;
  static constexpr size_t f32_end = p_out + (size_t)TM_D * TM_D * 4;
  static constexpr size_t w1_16 = align_up(f32_end, 256);
  static constexpr size_t p_out_16 = w1_16 + (size_t)TM_W1 * TM_D * 2;
  static constexpr size_t img_pg = align_up(p_out_16 + (size_t)TM_D * TM_D * 2, 1024);
  static constexpr size_t img_po = img_pg + (size_t)5 * TM_D * TM_D * 2;  // p_out as a 128 x 128 image
  static constexpr size_t end16 = img_po + (size_t)TM_D * TM_D * 2;
  static constexpr size_t bytes(int dtype) { return dtype == DT_F32 ? align_up(f32_end, 256) : align_up(end16, 256); }
};
// workspace of one call over P = B*N*N pairs (es = element size of the layer's type).  The channel
// planes of a, b and o are N rows of Np elements (16-bit modes: Np = N rounded up to 8, so that every
// row starts 16-byte aligned for the contraction's TMA loads; fp32 mode: Np = N).
//   xn  fp32 mode: [P][128] LayerNorm-in output, later norm_out's output (same place); 16-bit: none
//   h   fp32 mode: [P][640] projection p | g | g_out; 16-bit modes: [P][128] g_out only (the fused
//       projection kernel gates a and b in its epilogue and writes the output gate's projection)
//   ab  [2][B][128][N][Np]  gated + masked a, b, channel-major (es); fp32 mode: later p_out's output
//       [P][128] fp32
//   o   [B][128][N][Np]     contraction output, fp32, channel-major
//   blas                    fp32 mode: 32 MiB scratch handed to cuBLAS
struct TrimulWorkspace {
  size_t off_xn, off_h, off_ab, off_o, off_blas, total;
  int Np;
  static constexpr size_t BLAS_BYTES = 32ull << 20;
  __host__ __device__ static TrimulWorkspace make(int B, int N, int dtype) {
    TrimulWorkspace w{};
    const bool f32 = dtype == DT_F32;
    w.Np = f32 ? N : (N + 7) / 8 * 8;
    const size_t P = (size_t)B * N * N, Pp = (size_t)B * N * w.Np, es = f32 ? 4 : 2, A = 256;
    size_t o = 0;
    w.off_xn = o; o = align_up(o + (f32 ? P * TM_D * es : 0), A);
    w.off_h = o; o = align_up(o + P * (f32 ? TM_W1 : TM_D) * es, A);
    const size_t ab = 2 * Pp * TM_D * es, po = f32 ? P * TM_D * 4 : 0;
    w.off_ab = o; o = align_up(o + (ab > po ? ab : po), A);
    w.off_o = o; o = align_up(o + Pp * TM_D * 4, A);
    w.off_blas = o; o = align_up(o + (f32 ? BLAS_BYTES : 0), A);
    w.total = o;
    return w;
  }
};
struct TrimulArgs {
  const float* z; const float* mask; const unsigned char* packed;
  int B, N, outgoing, dtype, add_residual;
  float* out; unsigned char* ws;
  // optional (16-bit modes): the next module's LayerNorm of out, written in the layer's type, and from
  // its rounded values the next triangle attention's tri bias (fp32 weights [HEADS][128] -> fp16
  // [B][HEADS][N][N], pairs in ln_out's order)
  const float* ln_next_w; const float* ln_next_b; void* ln_out;
  const float* tb_next_w; void* tb_next;
};

// Byte offset of tri-bias element (q, k) of head h, batch b on the 16-bit path.
__host__ __device__ __forceinline__ size_t bias16_off(int q, int k, int b, int h, int B, int NT) {
  const size_t blk = (((size_t)(q >> 7) * B + b) * HEADS + h) * NT + (k >> 7);
  return blk * 32768 + (size_t)((k & 127) >> 3) * 2048 + (size_t)(q & 127) * 16 + (k & 7) * 2;
}

// Byte offset of V element (key, ch) inside a 128-key x 32-channel fp16 V image (MN-major).
__host__ __device__ __forceinline__ uint32_t vimg_off(uint32_t key, uint32_t ch) {
  return (ch >> 3) * 2048u + (key >> 3) * 128u + (key & 7u) * 16u + (ch & 7u) * 2u;
}

// Attention-oriented view of a [B][N][N][ch] tensor: element (b, a, c, ch) lives at
//   base + b * s_batch + (a - row0) * s_row + col(c) + ch,
//   col(c) = c * s_col                                         (cblk = 0)
//          = (c / cblk) * s_cblk + (c % cblk) * s_col           (columns in blocks of cblk)
// (starting node: s_row = N*ch, s_col = ch; ending node: s_row = ch, s_col = N*ch; a row-sharded
// residual stream kept as [P][rows][cols of rank p][ch] blocks: s_row = cblk*ch, s_col = ch,
// s_cblk = rows*cblk*ch).
// With a block table (tab != nullptr, device memory, N / cblk entries) block q starts at tab[q]
// elements from base instead of q * s_cblk: the blocks may then sit in other GPUs' memory mapped
// into this process (the peer-store exchange of the row-sharded layer).
struct View {
  long long s_batch, s_row, s_col;
  int row0;
  int cblk;
  long long s_cblk;
  const long long* tab;
};
__device__ __forceinline__ long long view_col(const View& v, int c) {
  if (!v.cblk) return (long long)c * v.s_col;
  const int q = c / v.cblk;
  return (v.tab ? __ldg(v.tab + q) : (long long)q * v.s_cblk) + (long long)(c - q * v.cblk) * v.s_col;
}

struct LayerArgs {
  int B, N, row_begin, row_end;
  float inf;
  const float* z; View zv;     // attention-oriented input
  const float* mask; View mv;  // attention-oriented mask (nullptr = ones)
  float* out; View ov;         // attention-oriented output
  int add_residual;
  const unsigned char* packed;
  unsigned char* ws;
  Workspace wl;
  int* status;                 // device status word
  int num_sms;                 // multiprocessors of the current device (persistent grids)
  // optional (16-bit path): this layer's LayerNorm output given by the caller (LN skipped; view in
  // 16-bit elements), and the next module's LayerNorm applied to the output, written in 16 bits
  const void* xn; View xnv;
  const float* ln_next_w; const float* ln_next_b;
  void* ln_out; View lnv;
  // optional (16-bit path, with xn): this layer's tri bias computed by the producer of xn, fp16
  // [B][HEADS][N][N] in natural units and the layer's attention orientation (the projection then skips
  // its own tri-bias dot); and, with ln_out, the next triangle attention's tri bias from the rounded
  // ln_out rows (fp32 weights [HEADS][128] -> fp16 [B][HEADS][N][N], pairs in ln_out's order)
  const void* tb_in;
  const float* tb_next_w; void* tb_next;
};

// Four per-head sums of one row spread over a warp (lane: partial p[h] of its channels).  Halves are
// exchanged first (xor 16: heads 0,1 | 2,3; xor 8: one head each), then three butterfly steps; every
// lane of group h (lanes 8h .. 8h + 7) ends with head h's total.
__device__ __forceinline__ float head_sums4(const float (&p)[HEADS], int lane) {
  const bool up16 = lane & 16, up8 = lane & 8;
  float k0 = up16 ? p[2] : p[0], k1 = up16 ? p[3] : p[1];
  k0 += __shfl_xor_sync(0xffffffffu, up16 ? p[0] : p[2], 16);
  k1 += __shfl_xor_sync(0xffffffffu, up16 ? p[1] : p[3], 16);
  float k = up8 ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, up8 ? k0 : k1, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  return k;
}

// launchers (return cudaGetLastError())
cudaError_t launch_pack_weights(const float* ln_w, const float* ln_b, const float* w_q, const float* w_k,
                                const float* w_v, const float* w_g, const float* g_bias, const float* w_b,
                                const float* w_o, int dtype, unsigned char* packed, cudaStream_t st);
cudaError_t launch_mask_prep(const LayerArgs& a, int dtype, cudaStream_t st);
cudaError_t launch_mask_prep_tc(const LayerArgs& a, cudaStream_t st);
cudaError_t launch_ln_proj_f32(const LayerArgs& a, cudaStream_t st);
cudaError_t launch_core_f32(const LayerArgs& a, cudaStream_t st);
cudaError_t launch_out_proj_f32(const LayerArgs& a, cudaStream_t st);
cudaError_t launch_ln_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st);
cudaError_t launch_core_tc(const LayerArgs& a, int dtype, cudaStream_t st);
cudaError_t launch_out_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st);
cudaError_t launch_peer_barrier(const unsigned long long* flag_ptrs, int rank, int world, unsigned epoch,
                                int* status, cudaStream_t st);
cudaError_t launch_peer_broadcast(const unsigned long long* dst_ptrs, int rank, int world, size_t offset, size_t bytes,
                                  int num_sms, cudaStream_t st);
cudaError_t launch_trimul_pack(const float* in_w, const float* in_b, const float* p_in, const float* g_in,
                               const float* out_w, const float* out_b, const float* p_out, const float* g_out,
                               int dtype, unsigned char* packed, cudaStream_t st);
// the layer: 4 kernels + 3 cuBLAS GEMMs; a cuBLAS failure returns cudaErrorUnknown with *blas_status set
cudaError_t launch_trimul(const TrimulArgs& a, cudaStream_t st, int* blas_status, const char** stage);
int* device_status_ptr();
int record_error(int code, const char* what, const char* detail);

}  // namespace triattn
