// Triangle multiplication, outgoing and incoming edges (boltz_mlx/layers/triangular_mult.py:10-178),
// forward only, on a B200:
//
//   16-bit modes:
//   F1  tm_proj_tc (tcgen05): LayerNorm-in -> UMMA with [p_in | g_in] (512 x 128) -> a = p sigmoid(g) m,
//       b likewise, stored channel-major [B][128][N][N] from the epilogue; xn [P][128] as a by-product
//   G1  cuBLAS GEMM   g_out = xn . g_out_w^T                              -> [P][128]
//   fp32 mode:
//   K1  LayerNorm-in, one warp per pair (two-pass fp32 statistics)      z fp32 -> xn [P][128]
//   G1  cuBLAS GEMM   h = xn . [p_in | g_in | g_out]^T                  -> h [P][640]
//   K2  gate + mask, transposed through shared memory to channel-major  -> a, b [B][128][N][N]
//   both:
//   G2  cuBLAS strided-batched GEMM, one N x N x N product per (batch, channel):
//         outgoing  o = a . b^T  (o[i,j] = sum_k a[i,k] b[j,k])
//         incoming  o = a^T . b  (o[i,j] = sum_k a[k,i] b[k,j])                -> o fp32 [B][128][N][N]
//   K3  LayerNorm-out over the 128 channels of each pair, transposed back to pair-major -> xn's place
//   G3  cuBLAS GEMM   y = norm_out(o) . p_out^T                           -> fp32 [P][128] (ab's place)
//   K4  out = z (residual) + y * sigmoid(g_out)
//
// The 16-bit modes keep xn, h, a, b and norm_out(o) in the layer's type with fp32 accumulation and an
// fp32 o (no overflow concern at any N, unlike an fp16 o); the fp32 mode runs every step in fp32 (the
// GEMMs in plain fp32, no TF32).  K1-K4 are HBM-bound streams (16-byte accesses, whole 128-byte rows
// per warp); the three GEMMs are plain library GEMMs.
#include <cstdint>
#include <cublas_v2.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <mutex>
#include <type_traits>

#include "sm100.cuh"
#include "triattn_internal.cuh"

namespace triattn {
namespace {

__device__ __forceinline__ float tm_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float tm_sigmoid(float x) { return 1.0f / (1.0f + __expf(-x)); }
// Batch, row and column of pair p of a [B][N][N] grid: 32-bit divides whenever p and N^2 fit in 32 bits
// (every size whose pair tensor fits in memory), the 64-bit ones otherwise.
struct PairIdx {
  long long b, row, col;
};
__device__ __forceinline__ PairIdx pair_idx(long long p, int N) {
  const unsigned long long nn = (unsigned long long)N * (unsigned long long)N;
  if ((unsigned long long)p < 0x100000000ull && nn < 0x100000000ull) {
    const uint32_t pu = (uint32_t)p, nu = (uint32_t)nn, bu = pu / nu, pp = pu - bu * nu, ru = pp / (uint32_t)N;
    return {(long long)bu, (long long)ru, (long long)(pp - ru * (uint32_t)N)};
  }
  const long long b = p / (long long)nn, pp = p - b * (long long)nn, r = pp / N;
  return {b, r, pp - r * N};
}

// the 16-bit kernels' gate.  fp16 layers: the approximate divide (2 ulp; 0 once the denominator passes
// 2^126, where the sigmoid is below 1e-38) in place of the IEEE one, whose refinement costs several
// instructions a call.  bf16 layers: sigmoid(x) = (1 + tanh(x / 2)) / 2 with the one-instruction MUFU
// tanh (absolute error about 2^-11 in tanh, 2^-12 in the sigmoid: an eighth of bf16's half-ulp at 1/2,
// so the bf16 rounding of the gated value dominates); one MUFU operation per element instead of two.
template <typename T>
__device__ __forceinline__ float tm_sigmoid_fast(float x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
    return fmaf(0.5f, t, 0.5f);
  } else {
    return __fdividef(1.0f, 1.0f + __expf(-x));
  }
}

// 4 / 2 consecutive elements of type T <-> float
template <typename T>
struct Ew;
template <>
struct Ew<float> {
  __device__ static float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
  __device__ static void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
  __device__ static float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
  __device__ static void st2(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
};
template <typename H>
struct Ew16 {
  __device__ static float4 ld4(const H* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = H16<H>::unpack(u.x), b = H16<H>::unpack(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  __device__ static void st4(H* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(H16<H>::pack(v.x, v.y), H16<H>::pack(v.z, v.w));
  }
  __device__ static float2 ld2(const H* p) { return H16<H>::unpack(*reinterpret_cast<const uint32_t*>(p)); }
  __device__ static void st2(H* p, float2 v) { *reinterpret_cast<uint32_t*>(p) = H16<H>::pack(v.x, v.y); }
};
template <>
struct Ew<__half> : Ew16<__half> {};
template <>
struct Ew<__nv_bfloat16> : Ew16<__nv_bfloat16> {};

// ---- K1: LayerNorm-in (reference norm_in, triangular_mult.py:28; eps 1e-5) ----------------------
template <typename T>
__global__ void __launch_bounds__(256) tm_ln_in_kernel(const float* __restrict__ z, const float* __restrict__ w,
                                                       const float* __restrict__ b, T* __restrict__ xn,
                                                       long long npairs) {
  const int lane = threadIdx.x & 31;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const float4 lw = reinterpret_cast<const float4*>(w)[lane], lb = reinterpret_cast<const float4*>(b)[lane];
  for (long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < npairs; p += nw) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(z + p * TM_D) + lane);
    const float mean = tm_warp_sum((v.x + v.y) + (v.z + v.w)) * (1.0f / TM_D);
    const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
    const float var = tm_warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3)) * (1.0f / TM_D);
    const float r = rsqrtf(var + LN_EPS);
    Ew<T>::st4(xn + p * TM_D + 4 * lane,
               make_float4(d0 * r * lw.x + lb.x, d1 * r * lw.y + lb.y, d2 * r * lw.z + lb.z, d3 * r * lw.w + lb.w));
  }
}

// ---- K2: a = p_a * sigmoid(g_a) * m, b = p_b * sigmoid(g_b) * m (triangular_mult.py:38-41), stored
//      channel-major: ab[s][bb][c][pp] (s = 0 a, 1 b; pp = pair index inside batch bb).  A CTA takes 64
//      consecutive pairs, a then b: warps read the h rows (lane = 4 channels), the gated values go
//      through shared memory [128 channels][64 pairs], then each warp writes channel rows of 64 pairs. --
constexpr int TM_GP = 64;  // pairs per CTA
template <typename T>
__global__ void __launch_bounds__(256) tm_gate_kernel(const T* __restrict__ h, const float* __restrict__ mask,
                                                      T* __restrict__ ab, long long npairs, long long nn, int B) {
  __shared__ float s[TM_D][TM_GP + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long p0 = (long long)blockIdx.x * TM_GP;
#pragma unroll 1
  for (int sel = 0; sel < 2; ++sel) {
    for (int pl = warp; pl < TM_GP; pl += 8) {
      const long long p = p0 + pl;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p < npairs) {
        const T* hr = h + p * TM_W1 + sel * TM_D + 4 * lane;
        const float m = mask ? mask[p] : 1.0f;
        const float4 pv = Ew<T>::ld4(hr), gv = Ew<T>::ld4(hr + 2 * TM_D);
        v = make_float4(pv.x * tm_sigmoid(gv.x) * m, pv.y * tm_sigmoid(gv.y) * m, pv.z * tm_sigmoid(gv.z) * m,
                        pv.w * tm_sigmoid(gv.w) * m);
      }
      s[4 * lane + 0][pl] = v.x;
      s[4 * lane + 1][pl] = v.y;
      s[4 * lane + 2][pl] = v.z;
      s[4 * lane + 3][pl] = v.w;
    }
    __syncthreads();
    // channel row c of the tile: lane writes pairs 2 lane, 2 lane + 1 (a warp covers 64 consecutive pairs)
    for (int c = warp; c < TM_D; c += 8) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const long long p = p0 + 2 * lane + e;
        if (p >= npairs) continue;
        const long long bb = p / nn, pp = p - bb * nn;
        ab[(((long long)sel * B + bb) * TM_D + c) * nn + pp] = static_cast<T>(s[c][2 * lane + e]);
      }
    }
    __syncthreads();
  }
}

// ---- K3: norm_out over the 128 channels of each pair (triangular_mult.py:49), from channel-major
//      fp32 o to pair-major T.  A CTA takes 32 consecutive pairs: warps read channel rows of 32 pairs
//      (128 bytes), then one warp per pair normalises (lane = 4 channels). -----------------------------
constexpr int TM_LP = 32;
template <typename T>
__global__ void __launch_bounds__(256) tm_ln_out_kernel(const float* __restrict__ o, const float* __restrict__ w,
                                                        const float* __restrict__ b, T* __restrict__ on,
                                                        long long npairs, long long nn) {
  __shared__ float s[TM_D][TM_LP + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long p0 = (long long)blockIdx.x * TM_LP;
  {
    const long long p = p0 + lane;
    const bool ok = p < npairs;
    const long long bb = ok ? p / nn : 0, pp = ok ? p - bb * nn : 0;
    const float* src = o + bb * TM_D * nn + pp;
    for (int c = warp; c < TM_D; c += 8) s[c][lane] = ok ? __ldcs(src + c * nn) : 0.0f;
  }
  __syncthreads();
  const float4 lw = reinterpret_cast<const float4*>(w)[lane], lb = reinterpret_cast<const float4*>(b)[lane];
  for (int pl = warp; pl < TM_LP; pl += 8) {
    const long long p = p0 + pl;
    if (p >= npairs) break;  // warp-uniform
    const float v0 = s[4 * lane][pl], v1 = s[4 * lane + 1][pl], v2 = s[4 * lane + 2][pl], v3 = s[4 * lane + 3][pl];
    const float mean = tm_warp_sum((v0 + v1) + (v2 + v3)) * (1.0f / TM_D);
    const float d0 = v0 - mean, d1 = v1 - mean, d2 = v2 - mean, d3 = v3 - mean;
    const float var = tm_warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3)) * (1.0f / TM_D);
    const float r = rsqrtf(var + LN_EPS);
    Ew<T>::st4(on + p * TM_D + 4 * lane,
               make_float4(d0 * r * lw.x + lb.x, d1 * r * lw.y + lb.y, d2 * r * lw.z + lb.z, d3 * r * lw.w + lb.w));
  }
}

// ---- K4: out = (z) + y * sigmoid(g_out) (triangular_mult.py:49 and the pairformer's residual) ----
template <typename T>
__global__ void __launch_bounds__(256) tm_out_kernel(const float* z, const float* __restrict__ y,
                                                     const T* __restrict__ gout, int g_stride, float* out,
                                                     long long n4, int add_residual) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const long long p = i >> 5, c = (i & 31) * 4;  // 32 float4 per pair
    const float4 yv = __ldcs(reinterpret_cast<const float4*>(y) + i);
    const float4 g = Ew<T>::ld4(gout + p * g_stride + c);
    float4 r = make_float4(yv.x * tm_sigmoid(g.x), yv.y * tm_sigmoid(g.y), yv.z * tm_sigmoid(g.z),
                           yv.w * tm_sigmoid(g.w));
    if (add_residual) {
      const float4 zv = reinterpret_cast<const float4*>(z)[i];  // out may alias z: read before write
      r.x += zv.x; r.y += zv.y; r.z += zv.z; r.w += zv.w;
    }
    reinterpret_cast<float4*>(out)[i] = r;
  }
}

// ---- F1 (16-bit modes): fused LayerNorm-in + [p_in | g_in | g_out] projection + gate/mask epilogue --
// Persistent, one CTA per SM (512 threads), the 160 KB operand image of [p_in | g_in | g_out] loaded once.
// Tile = 128 consecutive pairs.  Per tile: LayerNorm (warp w: pairs 8w..8w+7, lane: channels
// 4 lane..+3) into a 128-byte-swizzled operand image; UMMA D[128 x 512] = xn [p_a | g_a | p_b | g_b]^T in
// two N = 256 halves (TMEM columns 0..255 | 256..511, one commit each); epilogue in three phases, warp
// (quad, tt) taking TMEM lanes 32 quad.. and channels 32 tt..: (a) a = p_a sigmoid(g_a) m into the
// channel-major a planes (a warp's 32 lanes are 32 consecutive pairs of one channel row: 64-byte runs);
// once every warp has read the a columns, the output gate's projection xn g_out^T (N = 128) runs into
// columns 0..127 while (b) gates b; (c) the output gate's projection (pre-sigmoid, 16-bit) into g_out
// [P][128] for the tail.  The LayerNorm of tile it + 1 runs while the MMA of tile it executes (two
// operand images), as in the attention projection kernel.
constexpr int TP_THREADS = 512;
constexpr int TP_W_BYTES = 5 * TM_D * TM_D * 2;  // 640 x 128 16-bit image
constexpr int TP_A_BYTES = TILE * TM_D * 2;      // one 128-pair LayerNorm image
constexpr int TP_SMEM = TP_W_BYTES + 2 * TP_A_BYTES + 64;
static_assert(TP_SMEM <= 232448, "projection shared memory");

template <typename T>
__global__ void __launch_bounds__(TP_THREADS, 1)
    tm_proj_tc_kernel(const float* __restrict__ z, const float* __restrict__ mask, const unsigned char* __restrict__ packed,
                      T* __restrict__ gout, T* __restrict__ ab, long long npairs, int N, int Np, int B, int* status) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sW = smem;
  unsigned char* sA = smem + TP_W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TP_W_BYTES + 2 * TP_A_BYTES);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);
  uint64_t* bar_w = bars;
  uint64_t* bar_mma = bars + 1;   // [3]: a half, b half, output gate
  uint64_t* bar_adone = bars + 4;  // every warp has read the a half's columns
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long ntiles = (npairs + TILE - 1) / TILE;
  const long long plane = (long long)N * Np;
  const float* Pf = reinterpret_cast<const float*>(packed);
  if ((smem_u32(sA) & 1023u) != 0) {  // the swizzled image needs a 1024-byte aligned base (CTA-uniform)
    if (tid == 0) atomicCAS(status, 0, (int)DEV_BAD_ALIGN);
    return;
  }
  if (tid == 0) {
    mbar_init(bar_w, 1);
    for (int i = 0; i < 3; ++i) mbar_init(bar_mma + i, 1);
    mbar_init(bar_adone, TP_THREADS / 32);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (tid == 0 && (long long)blockIdx.x < ntiles) {
    mbar_arrive_expect_tx(bar_w, TP_W_BYTES);
    bulk_g2s(sW, packed + TrimulPacked::img_pg, TP_W_BYTES, bar_w);
  }
  const float4 lw = reinterpret_cast<const float4*>(Pf + TrimulPacked::in_w / 4)[lane];
  const float4 lb = reinterpret_cast<const float4*>(Pf + TrimulPacked::in_b / 4)[lane];
  auto load_rows = [&](long long tile, float4 (&xv)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const long long p = tile * TILE + warp * 8 + i;
      xv[i] = p < npairs ? __ldcs(reinterpret_cast<const float4*>(z + p * TM_D) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto ln_tile = [&](int it, const float4 (&xv)[8]) {
    unsigned char* sAi = sA + (it & 1) * TP_A_BYTES;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = warp * 8 + i;
      const float4 v = xv[i];
      const float mean = tm_warp_sum((v.x + v.y) + (v.z + v.w)) * (1.0f / TM_D);
      const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
      const float var = tm_warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3)) * (1.0f / TM_D);
      const float rs = rsqrtf(var + LN_EPS);
      const uint2 pk = make_uint2(H16<T>::pack(d0 * rs * lw.x + lb.x, d1 * rs * lw.y + lb.y),
                                  H16<T>::pack(d2 * rs * lw.z + lb.z, d3 * rs * lw.w + lb.w));
      *reinterpret_cast<uint2*>(sAi + sw128_off(r, 4 * lane, TP_A_BYTES / 2)) = pk;
    }
  };
  // rows [row0, row0 + N) of the weight image against image it & 1 into TMEM column col0 (one thread)
  auto mma_rows = [&](int it, int row0, int col0, auto n_const) {
    constexpr int NN = decltype(n_const)::value;
    unsigned char* sAi = sA + (it & 1) * TP_A_BYTES;
    constexpr uint32_t idesc = make_idesc_f16(128, NN, H16<T>::is_bf16, 0, 0);
#pragma unroll
    for (int ks = 0; ks < TM_D / 16; ++ks) {
      const uint64_t ad = smem_desc_sw128(smem_u32(sAi) + (ks / 4) * (TP_A_BYTES / 2) + (ks % 4) * 32);
      const uint64_t bd = smem_desc_noswizzle(smem_u32(sW) + (row0 / 8) * (16 * TM_D) + ks * 256, 128, 16 * TM_D);
      umma_ss(tbase + col0, ad, bd, idesc, ks > 0 ? 1u : 0u);
    }
  };
  auto issue_mma = [&](int it) {
    if (tid == 0) {
      if (it == 0) mbar_wait(bar_w, 0, status, DEV_TIMEOUT_TMA);
      tc_fence_after();
      mma_rows(it, 0, 0, std::integral_constant<int, 256>{});  // p_a | g_a
      umma_commit(bar_mma + 0);
      mma_rows(it, 256, 256, std::integral_constant<int, 256>{});  // p_b | g_b
      umma_commit(bar_mma + 1);
    }
  };
  auto epilogue = [&](int it, long long tile) {
    const int quad = warp & 3, tt = warp >> 2;
    const long long p = tile * TILE + quad * 32 + lane;
    const bool valid = p < npairs;
    const float m = valid ? (mask ? mask[p] : 1.0f) : 0.0f;
    const PairIdx pi = pair_idx(valid ? p : 0, N);
    const long long bb = pi.b, prow = pi.row, pcol = pi.col;
    // channels 32 tt .. 32 tt + 31 of a (sel 0) or b (sel 1): p at TMEM column colp + c, g at colg + c
    auto gate = [&](int sel, int colp, int colg) {
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        const int c = 32 * tt + 16 * h2;
        uint32_t pv[16], gv[16];
        tmem_ld16(tmem_addr(tbase, quad * 32, colp + c), pv);
        tmem_ld16(tmem_addr(tbase, quad * 32, colg + c), gv);
        tmem_ld_wait();
        tmem_regs_ready(pv);
        tmem_regs_ready(gv);
        if (valid) {
          T* dst = ab + ((long long)(sel * B + bb) * TM_D + c) * plane + prow * Np + pcol;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            dst[j * plane] = static_cast<T>(__uint_as_float(pv[j]) * tm_sigmoid_fast<T>(__uint_as_float(gv[j])) * m);
        }
      }
    };
    mbar_wait(bar_mma + 0, it & 1, status, DEV_TIMEOUT_MMA);
    __syncwarp();
    tc_fence_after();
    gate(0, 0, 128);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_adone);
    if (tid == 0) {  // the a columns are free: the output gate's projection into columns 0..127
      mbar_wait(bar_adone, it & 1, status, DEV_TIMEOUT_SYNC);
      tc_fence_after();
      mma_rows(it, 512, 0, std::integral_constant<int, 128>{});
      umma_commit(bar_mma + 2);
    }
    mbar_wait(bar_mma + 1, it & 1, status, DEV_TIMEOUT_MMA);
    __syncwarp();
    tc_fence_after();
    gate(1, 256, 384);
    mbar_wait(bar_mma + 2, it & 1, status, DEV_TIMEOUT_MMA);
    __syncwarp();
    tc_fence_after();
    {
      uint32_t gv[32];
      tmem_ld32(tmem_addr(tbase, quad * 32, 32 * tt), gv);
      tmem_ld_wait();
      tmem_regs_ready(gv);
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(gout + p * TM_D + 32 * tt);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(H16<T>::pack(__uint_as_float(gv[8 * q + 0]), __uint_as_float(gv[8 * q + 1])),
                              H16<T>::pack(__uint_as_float(gv[8 * q + 2]), __uint_as_float(gv[8 * q + 3])),
                              H16<T>::pack(__uint_as_float(gv[8 * q + 4]), __uint_as_float(gv[8 * q + 5])),
                              H16<T>::pack(__uint_as_float(gv[8 * q + 6]), __uint_as_float(gv[8 * q + 7])));
      }
    }
  };
  // the z rows of tile t (128 consecutive pairs: one contiguous 64 KB run) pulled into L2 two tiles ahead
  // of their register loads, by one thread (the bulk-copy unit takes one request at a time)
  auto prefetch_tile = [&](long long t) {
    if (tid == 32 && t < ntiles) {
      const long long p0 = t * TILE, np = npairs - p0 < TILE ? npairs - p0 : TILE;
      prefetch_l2_bulk(z + p0 * TM_D, (uint32_t)(np * TM_D * 4));
    }
  };
  float4 xv[8];
  long long tile = blockIdx.x;
  if (tile < ntiles) {
    prefetch_tile(tile + 2 * gridDim.x);
    prefetch_tile(tile + 3 * gridDim.x);
    load_rows(tile, xv);
    ln_tile(0, xv);
    if (tile + gridDim.x < ntiles) load_rows(tile + gridDim.x, xv);
    fence_proxy_async_smem();
    __syncthreads();
    issue_mma(0);
  }
  for (int it = 0; tile < ntiles; tile += gridDim.x, ++it) {
    const long long nxt = tile + gridDim.x;
    prefetch_tile(tile + 4 * gridDim.x);
    if (nxt < ntiles) {
      ln_tile(it + 1, xv);  // overlaps the MMA of this tile
      if (nxt + gridDim.x < ntiles) load_rows(nxt + gridDim.x, xv);
      fence_proxy_async_smem();
    }
    epilogue(it, tile);
    tc_fence_before();
    __syncthreads();  // image it + 1 complete; every epilogue done with TMEM
    tc_fence_after();
    if (nxt < ntiles) issue_mma(it + 1);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// ---- G2 (16-bit modes): the per-channel contraction on the tensor cores ---------------------------
// o[pl][i][j] = sum_k A[i][k] B[j][k] for every plane pl = (batch, channel) (triangular_mult.py:43-47):
//   outgoing  A[i][k] = a[pl][i][k], B[j][k] = b[pl][j][k]  (K-major operands: k contiguous)
//   incoming  A[i][k] = a[pl][k][i], B[j][k] = b[pl][k][j]  (MN-major operands: i / j contiguous)
// a, b: [planes][N][Np] 16-bit, read by TMA through 3-D tensor maps (x = column, y = row, z = plane;
// 128-byte swizzle; zero fill past N, so ragged edges and the K tail need no padding in memory).
// o: fp32 [planes][N][Np].  Persistent, one CTA per SM: warp 0 lane 0 issues the TMA loads, warp 1
// lane 0 the MMAs (UMMA M = 128, N = 256, fp32 accumulation in TMEM), the other warps are the epilogue
// (one thread per output row; TMEM lane quadrant = warp % 4).  K runs in blocks of 64 through a ring of
// shared-memory stages.  Two tile shapes:
//   BM = 128: tile 128 x 256, 4 stages of 48 KB, two accumulators (2 x 256 TMEM columns) so that the
//             epilogue of one tile overlaps the main loop of the next;
//   BM = 256: tile 256 x 256 (two M = 128 MMAs share each B block: 2/3 of the operand bytes per flop),
//             3 stages of 64 KB, one accumulator of 512 columns; the producer prefetches the next tile's
//             first stages while the 8 epilogue warps drain it.
// Tiles are numbered plane-major (then row block, then column block), so the CTAs running at the same
// time share a plane's a and b in L2.
template <int BM>
struct CtCfg {
  static constexpr int BN = 256, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = BM == 128 ? 4 : 3;
  static constexpr int ACCS = BM == 128 ? 2 : 1;  // accumulators of BM / 128 x 256 TMEM columns
  static constexpr int EPI_WARPS = BM / 32;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int SMEM = 1024 + STAGES * STAGE + 256;  // + alignment slack + barriers
  static_assert(SMEM <= 232448, "contraction shared memory");
  static_assert(ACCS * (BM / 128) * 256 == 512, "TMEM columns");
};
#ifndef TRIATTN_CT_BM
#define TRIATTN_CT_BM 128
#endif
constexpr int CT_BM = TRIATTN_CT_BM;  // tile shape used by the layer

template <typename T, bool MN, int BM>
__global__ void __launch_bounds__(CtCfg<BM>::THREADS, 1)
    tm_contract_tc_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                          float* __restrict__ o, int N, int Np, int planes, int* status) {
  using C = CtCfg<BM>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1024-aligned stages
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);  // [STAGES] loads landed
  uint64_t* empty = full + C::STAGES;                                          // [STAGES] MMAs done reading
  uint64_t* acc_full = empty + C::STAGES;                                      // [ACCS] accumulator complete
  uint64_t* acc_empty = acc_full + C::ACCS;                                    // [ACCS] accumulator read out
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + C::ACCS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtn = (N + BM - 1) / BM, ntn = (N + C::BN - 1) / C::BN, nk = (N + C::BK - 1) / C::BK;
  const int ntiles = planes * mtn * ntn;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < C::ACCS; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, C::EPI_WARPS);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  auto coords = [&](int t, int& pl, int& m0, int& n0) {
    const int r = t / ntn;
    n0 = (t - r * ntn) * C::BN;
    pl = r / mtn;
    m0 = (r - pl * mtn) * BM;
  };
  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      int it = 0;  // k blocks issued over all tiles
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        int pl, m0, n0;
        coords(t, pl, m0, n0);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % C::STAGES;
          mbar_wait(empty + st, ((it / C::STAGES) & 1) ^ 1, status, DEV_TIMEOUT_MMA);
          unsigned char* sa = smem + st * C::STAGE;
          unsigned char* sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(full + st, C::STAGE);
          const int k0 = kb * C::BK;
          if constexpr (!MN) {
            tma_load_3d(sa, &tma, k0, m0, pl, full + st);  // BM rows x 64 k
            tma_load_3d(sb, &tmb, k0, n0, pl, full + st);  // 256 rows x 64 k
          } else {
#pragma unroll
            for (int q = 0; q < BM / 64; ++q) tma_load_3d(sa + q * 8192, &tma, m0 + 64 * q, k0, pl, full + st);
#pragma unroll
            for (int q = 0; q < C::BN / 64; ++q) tma_load_3d(sb + q * 8192, &tmb, n0 + 64 * q, k0, pl, full + st);
          }
        }
      }
      // copies still in flight after an error: wait (bounded) for the last load of every stage
      for (int st = 0; st < C::STAGES && st < it; ++st) {
        const int last = it - 1 - ((it - 1 - st) % C::STAGES);
        mbar_wait_drain(full + st, (last / C::STAGES) & 1, 200000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: per K step of 16, BM / 128 MMAs of 128 x 256 sharing the B block ----
      constexpr uint32_t idesc = make_idesc_f16(128, C::BN, H16<T>::is_bf16, MN ? 1 : 0, MN ? 1 : 0);
      int it = 0, tl = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
        const int acc = tl % C::ACCS;
        mbar_wait(acc_empty + acc, ((tl / C::ACCS) & 1) ^ 1, status, DEV_TIMEOUT_MMA);
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % C::STAGES;
          mbar_wait(full + st, (it / C::STAGES) & 1, status, DEV_TIMEOUT_TMA);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + st * C::STAGE), sb = sa + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < C::BK / 16; ++ks) {
            const uint64_t bd = MN ? smem_desc_sw128_mn(sb + ks * 2048, 8192) : smem_desc_sw128(sb + ks * 32);
#pragma unroll
            for (int h = 0; h < BM / 128; ++h) {
              const uint32_t sah = sa + h * 16384;  // rows 128 h.. of the A block (either layout)
              const uint64_t ad = MN ? smem_desc_sw128_mn(sah + ks * 2048, 8192) : smem_desc_sw128(sah + ks * 32);
              umma_ss(tbase + (acc + h) * 256, ad, bd, idesc, (kb | ks) ? 1u : 0u);
            }
          }
          umma_commit(empty + st);  // the stage is free once these MMAs have read it
        }
        umma_commit(acc_full + acc);
      }
    }
  } else {
    // ---- epilogue: one thread per output row, fp32 stores of 32 columns at a time ----
    const int e = warp - 2, q = warp & 3, h = e >> 2;  // rows m0 + 128 h + 32 q + lane
    int tl = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
      int pl, m0, n0;
      coords(t, pl, m0, n0);
      const int acc = tl % C::ACCS;
      mbar_wait(acc_full + acc, (tl / C::ACCS) & 1, status, DEV_TIMEOUT_MMA);
      __syncwarp();
      tc_fence_after();
      const int i = m0 + 128 * h + 32 * q + lane;
      float* orow = o + ((long long)pl * N + (i < N ? i : 0)) * Np;
#pragma unroll 1
      for (int c = 0; c < C::BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_addr(tbase + (acc + h) * 256, 32 * q, 32 * c), v);
        tmem_ld_wait();
        tmem_regs_ready(v);
        const int j0 = n0 + 32 * c;
        if (i < N) {
#pragma unroll
          for (int e4 = 0; e4 < 32; e4 += 4)
            if (j0 + e4 < Np)
              *reinterpret_cast<float4*>(orow + j0 + e4) = make_float4(
                  __uint_as_float(v[e4]), __uint_as_float(v[e4 + 1]), __uint_as_float(v[e4 + 2]), __uint_as_float(v[e4 + 3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// ---- T1 (16-bit modes): the tail in one kernel: norm_out + p_out MMA + output gate + residual ------
// Tile = 128 consecutive pairs, one per CTA, 256 threads, three CTAs per SM.
//   norm_out: thread (pair r = tid % 128, half = tid / 128) holds channels 64 half.. of o for its pair
//     in registers (a warp's loads are 128-byte runs: 32 consecutive pairs of one channel row); the
//     two halves' sums meet in shared memory; two-pass fp32 statistics as the reference; the 16-bit
//     result goes into a K-major operand image.
//   MMA: D[128 x 128] = norm_out(o) . p_out^T (TMEM 128 columns).
//   epilogue: the accumulator is staged through shared memory (rows of 132 floats, over the operand
//     images), then warp w streams rows 16w..16w+15 whole: out = z + y * sigmoid(g_out).
constexpr int TT_THREADS = 256;
constexpr int TT_STAGE_LD = TM_D + 4;
constexpr int TT_SMEM_BODY = TILE * TT_STAGE_LD * 4;  // 67584 B, covers the two 32 KB operand images
constexpr int TT_SMEM = TT_SMEM_BODY + 2 * 2 * TILE * 4 + 64;

template <typename T, bool LN_NEXT, bool TB>
__global__ void __launch_bounds__(TT_THREADS, 3)
    tm_tail_tc_kernel(const float* __restrict__ o, const unsigned char* __restrict__ packed, const T* __restrict__ gout,
                      const float* z, float* out, long long npairs, int N, int Np, int add_residual,
                      const float* __restrict__ ln_w, const float* __restrict__ ln_b, T* __restrict__ ln_out,
                      const float* __restrict__ tb_w, __half* __restrict__ tb_out, int* status) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sA = smem;
  unsigned char* sW = smem + 32768;
  float* stage = reinterpret_cast<float*>(smem);  // after the MMA
  float* red = reinterpret_cast<float*>(smem + TT_SMEM_BODY);  // [2 stats][2 halves][128 pairs]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TT_SMEM_BODY + 2 * 2 * TILE * 4);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long p0 = (long long)blockIdx.x * TILE;
  const float* Pf = reinterpret_cast<const float*>(packed);
  if (tid == 0) {
    mbar_init(bars + 0, 1);
    mbar_init(bars + 1, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (tid == 0) {
    mbar_arrive_expect_tx(bars + 0, 32768);
    bulk_g2s(sW, packed + TrimulPacked::img_po, 32768, bars + 0);
  }
  // the epilogue's row streams (z residual, output gate) pulled into L2 while norm_out and the MMA run:
  // 128 consecutive pairs are one contiguous run in each
  if (tid == 32 && p0 < npairs) {
    const long long np = npairs - p0 < TILE ? npairs - p0 : TILE;
    if (add_residual) prefetch_l2_bulk(z + p0 * TM_D, (uint32_t)(np * TM_D * 4));
    prefetch_l2_bulk(gout + p0 * TM_D, (uint32_t)(np * TM_D * sizeof(T)));
  }
  // ---- norm_out of pair r over channels 64 half .. 64 half + 63 ----
  {
    const int r = tid & (TILE - 1), half = tid >> 7;
    const long long p = p0 + r;
    const bool valid = p < npairs;
    const long long nn = (long long)N * N, plane = (long long)N * Np;
    const long long bb = valid ? p / nn : 0, pp = valid ? p - bb * nn : 0;
    const long long prow = pp / N;
    const float* src = o + (bb * TM_D + 64 * half) * plane + prow * Np + (pp - prow * N);
    float v[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) v[d] = valid ? __ldcs(src + d * plane) : 0.0f;
    // statistics and affine on packed fp32 pairs (even, odd channel): the same roundings, in the same
    // order, as scalar even / odd partial sums, at half the instructions
    const float2* v2 = reinterpret_cast<const float2*>(v);
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int d = 0; d < 32; ++d) s2 = __fadd2_rn(s2, v2[d]);
    red[half * TILE + r] = s2.x + s2.y;
    __syncthreads();
    const float mean = (red[r] + red[TILE + r]) * (1.0f / TM_D);
    const float2 nmean = make_float2(-mean, -mean);
    float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      const float2 e = __fadd2_rn(v2[d], nmean);
      q2 = __ffma2_rn(e, e, q2);
    }
    red[2 * TILE + half * TILE + r] = q2.x + q2.y;
    __syncthreads();
    const float var = (red[2 * TILE + r] + red[3 * TILE + r]) * (1.0f / TM_D);
    const float rs = rsqrtf(var + LN_EPS);
    const float2 rs2 = make_float2(rs, rs);
    const float4* lw4 = reinterpret_cast<const float4*>(Pf + TrimulPacked::out_w / 4 + 64 * half);
    const float4* lb4 = reinterpret_cast<const float4*>(Pf + TrimulPacked::out_b / 4 + 64 * half);
#pragma unroll
    for (int d = 0; d < 64; d += 8) {
      uint32_t w4[4];
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const float4 w = __ldg(lw4 + (d + 2 * e) / 4), bq = __ldg(lb4 + (d + 2 * e) / 4);
        const float2 n0 = __ffma2_rn(__fmul2_rn(__fadd2_rn(v2[(d + 2 * e) / 2], nmean), rs2), make_float2(w.x, w.y),
                                     make_float2(bq.x, bq.y));
        const float2 n1 = __ffma2_rn(__fmul2_rn(__fadd2_rn(v2[(d + 2 * e) / 2 + 1], nmean), rs2), make_float2(w.z, w.w),
                                     make_float2(bq.z, bq.w));
        w4[e] = H16<T>::pack(n0.x, n0.y);
        w4[e + 1] = H16<T>::pack(n1.x, n1.y);
      }
      *reinterpret_cast<uint4*>(sA + img_off(r, 64 * half + d, TM_D)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    mbar_wait(bars + 0, 0, status, DEV_TIMEOUT_TMA);
    tc_fence_after();
    constexpr uint32_t idesc = make_idesc_f16(128, 128, H16<T>::is_bf16, 0, 0);
#pragma unroll
    for (int ks = 0; ks < TM_D / 16; ++ks) {
      const uint64_t ad = smem_desc_noswizzle(smem_u32(sA) + ks * 256, 128, 16 * TM_D);
      const uint64_t bd = smem_desc_noswizzle(smem_u32(sW) + ks * 256, 128, 16 * TM_D);
      umma_ss(tbase, ad, bd, idesc, ks > 0 ? 1u : 0u);
    }
    umma_commit(bars + 1);
  }
  mbar_wait(bars + 1, 0, status, DEV_TIMEOUT_MMA);  // MMA done: the operand images are free for staging
  __syncwarp();
  tc_fence_after();
  {
    const int quad = warp & 3, part = warp >> 2;
    float* srow = stage + (quad * 32 + lane) * TT_STAGE_LD + 64 * part;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      uint32_t acc[32];
      tmem_ld32(tmem_addr(tbase, quad * 32, 64 * part + 32 * h2), acc);
      tmem_ld_wait();
      tmem_regs_ready(acc);
#pragma unroll
      for (int d = 0; d < 32; d += 4)
        *reinterpret_cast<float4*>(srow + 32 * h2 + d) =
            make_float4(__uint_as_float(acc[d]), __uint_as_float(acc[d + 1]), __uint_as_float(acc[d + 2]),
                        __uint_as_float(acc[d + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  // ---- rows 16 warp .. 16 warp + 15: out = z + y * sigmoid(g_out), lane = channels 4 lane.. (and
  //      the next module's LayerNorm of the new row, two-pass fp32 statistics, one 16-bit rounding) ----
  float4 nw = make_float4(0.f, 0.f, 0.f, 0.f), nb = nw;
  if constexpr (LN_NEXT) {
    nw = reinterpret_cast<const float4*>(ln_w)[lane];
    nb = reinterpret_cast<const float4*>(ln_b)[lane];
  }
  // the next triangle attention's tri bias from the rounded LayerNorm rows: lane 8 hh + i keeps head hh
  // of rows 16 warp + i (tbk0) and 16 warp + 8 + i (tbk1)
  constexpr bool tb_on = LN_NEXT && TB;
  float tbk0 = 0.f, tbk1 = 0.f;
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int r = 16 * warp + i;
    const long long p = p0 + r;
    if (p >= npairs) break;  // warp-uniform
    const float4 y = *reinterpret_cast<const float4*>(stage + r * TT_STAGE_LD + 4 * lane);
    const float4 g = Ew<T>::ld4(gout + p * TM_D + 4 * lane);
    float4 res = make_float4(y.x * tm_sigmoid_fast<T>(g.x), y.y * tm_sigmoid_fast<T>(g.y), y.z * tm_sigmoid_fast<T>(g.z),
                             y.w * tm_sigmoid_fast<T>(g.w));
    if (add_residual) {
      const float4 zv = reinterpret_cast<const float4*>(z + p * TM_D)[lane];  // out may alias z
      res.x += zv.x; res.y += zv.y; res.z += zv.z; res.w += zv.w;
    }
    reinterpret_cast<float4*>(out + p * TM_D)[lane] = res;
    if constexpr (LN_NEXT) {
      const float mean = tm_warp_sum((res.x + res.y) + (res.z + res.w)) * (1.0f / TM_D);
      const float d0 = res.x - mean, d1 = res.y - mean, d2 = res.z - mean, d3 = res.w - mean;
      const float var = tm_warp_sum((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3)) * (1.0f / TM_D);
      const float rs = rsqrtf(var + LN_EPS);
      const float4 ln4 = make_float4(d0 * rs * nw.x + nb.x, d1 * rs * nw.y + nb.y, d2 * rs * nw.z + nb.z,
                                     d3 * rs * nw.w + nb.w);
      const uint2 pk = make_uint2(H16<T>::pack(ln4.x, ln4.y), H16<T>::pack(ln4.z, ln4.w));
      *reinterpret_cast<uint2*>(ln_out + p * TM_D + 4 * lane) = pk;
      if constexpr (tb_on) {
        // reference _LN_EPI_TB (kernels_nax3.py:104-143): fp32 sums of the rounded LayerNorm values
        const float2 h01 = H16<T>::unpack(pk.x), h23 = H16<T>::unpack(pk.y);
        float pp[HEADS];
#pragma unroll
        for (int hh = 0; hh < HEADS; ++hh) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(tb_w + hh * TM_D) + lane);
          pp[hh] = h01.x * w.x + h01.y * w.y + h23.x * w.z + h23.y * w.w;
        }
        const float k = head_sums4(pp, lane);
        if ((lane & 7) == (i & 7)) {
          if (i < 8) tbk0 = k;
          else tbk1 = k;
        }
      }
    }
  }
  if constexpr (tb_on) {
    // fp16 [B][HEADS][N][N]: pair p of batch bb -> (bb * HEADS + hh) * nn + (p - bb * nn)
    const int hh = lane >> 3;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const long long p = p0 + 16 * warp + 8 * h + (lane & 7);
      if (p < npairs) {
        const long long nn = (long long)N * N, bb = p / nn;
        tb_out[(bb * HEADS + hh) * nn + (p - bb * nn)] = __float2half_rn(h ? tbk1 : tbk0);
      }
    }
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 128);
}

// ---- weight packing ------------------------------------------------------------------------------
template <typename T>
__global__ void tm_pack_kernel(const float* in_w, const float* in_b, const float* p_in, const float* g_in,
                               const float* out_w, const float* out_b, const float* p_out, const float* g_out,
                               unsigned char* packed, int with16) {
  float* f = reinterpret_cast<float*>(packed);
  const int stride = gridDim.x * blockDim.x;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TM_W1 * TM_D; i += stride) {
    const int r = i / TM_D;
    // W1 rows: p_in (256) | g_in (256) | g_out (128)
    const float v = r < 2 * TM_D ? p_in[i] : (r < 4 * TM_D ? g_in[i - 2 * TM_D * TM_D] : g_out[i - 4 * TM_D * TM_D]);
    f[TrimulPacked::w1 / 4 + i] = v;
    if (with16) {
      reinterpret_cast<T*>(packed + TrimulPacked::w1_16)[i] = static_cast<T>(v);
      // image row of W1 row r: p_in[0:128] | g_in[0:128] | p_in[128:256] | g_in[128:256] | g_out
      const int ri = r < 2 * TM_D ? (r < TM_D ? r : r + TM_D) : (r < 4 * TM_D ? (r < 3 * TM_D ? r - TM_D : r) : r);
      reinterpret_cast<T*>(packed + TrimulPacked::img_pg)[img_off(ri, i % TM_D, TM_D) / 2] = static_cast<T>(v);
      if (r < TM_D)
        reinterpret_cast<T*>(packed + TrimulPacked::img_po)[img_off(r, i % TM_D, TM_D) / 2] = static_cast<T>(p_out[i]);
    }
    if (r < TM_D) {
      f[TrimulPacked::p_out / 4 + i] = p_out[i];
      if (with16) reinterpret_cast<T*>(packed + TrimulPacked::p_out_16)[i] = static_cast<T>(p_out[i]);
    }
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TM_D; i += stride) {
    f[TrimulPacked::in_w / 4 + i] = in_w[i];
    f[TrimulPacked::in_b / 4 + i] = in_b[i];
    f[TrimulPacked::out_w / 4 + i] = out_w[i];
    f[TrimulPacked::out_b / 4 + i] = out_b[i];
  }
}

// ---- cuBLAS: one handle per device, created on first use ------------------------------------------
cublasHandle_t blas_handle(int* err) {
  static std::mutex mu;
  static cublasHandle_t handles[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = -1;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!handles[dev]) {
    cublasHandle_t h = nullptr;
    const cublasStatus_t s = cublasCreate(&h);
    if (s != CUBLAS_STATUS_SUCCESS) {
      *err = (int)s;
      return nullptr;
    }
    handles[dev] = h;
  }
  return handles[dev];
}

int grid_for(long long work, int per_block, int cap) {
  const long long g = (work + per_block - 1) / per_block;
  return (int)(g < cap ? (g < 1 ? 1 : g) : cap);
}

// TMA descriptor of the a or b planes: [planes][N][Np] 16-bit, x = column (contiguous), y = row,
// z = plane, box (64, box_y, 1), 128-byte swizzle, zero fill outside [0, N) x [0, N).
// cuTensorMapEncodeTiled comes from the driver through the runtime's entry-point query (no libcuda link).
cudaError_t encode_planes(CUtensorMap* m, const void* base, bool bf16, int N, int Np, int planes, int box_y) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)N, (cuuint64_t)planes};
  const cuuint64_t strides[2] = {(cuuint64_t)Np * 2, (cuuint64_t)N * Np * 2};
  const cuuint32_t box[3] = {64u, (cuuint32_t)box_y, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// G2 launch: tensor maps of the a and b planes (outgoing: K-major boxes of 64 k x BM (a) / 256 (b) rows;
// incoming: MN-major boxes of 64 columns x 64 k), one persistent CTA per SM.
template <typename T, int BM>
cudaError_t launch_contract(const T* ab, bool bf16, bool outgoing, float* o, int N, int Np, int planes, int sms,
                            int* status, cudaStream_t st) {
  using C = CtCfg<BM>;
  CUtensorMap ma, mb;
  cudaError_t e;
  if ((e = encode_planes(&ma, ab, bf16, N, Np, planes, outgoing ? BM : C::BK)) != cudaSuccess) return e;
  if ((e = encode_planes(&mb, ab + (size_t)planes * N * Np, bf16, N, Np, planes, outgoing ? C::BN : C::BK)) !=
      cudaSuccess)
    return e;
  const int ctiles = planes * ((N + BM - 1) / BM) * ((N + C::BN - 1) / C::BN);
  const int grid = ctiles < sms ? ctiles : sms;
  if (outgoing) {
    cudaFuncSetAttribute(tm_contract_tc_kernel<T, false, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    tm_contract_tc_kernel<T, false, BM><<<grid, C::THREADS, C::SMEM, st>>>(ma, mb, o, N, Np, planes, status);
  } else {
    cudaFuncSetAttribute(tm_contract_tc_kernel<T, true, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    tm_contract_tc_kernel<T, true, BM><<<grid, C::THREADS, C::SMEM, st>>>(ma, mb, o, N, Np, planes, status);
  }
  return cudaGetLastError();
}

// 16-bit modes: F1 projection -> G2 contraction -> T1 tail, all hand-written tcgen05 kernels.
template <typename T>
cudaError_t trimul_run16(const TrimulArgs& a, cudaStream_t st, const char** stage) {
  const TrimulWorkspace wl = TrimulWorkspace::make(a.B, a.N, a.dtype);
  const int N = a.N, Np = wl.Np, planes = a.B * TM_D;
  const long long P = (long long)a.B * N * N;
  T* gout = reinterpret_cast<T*>(a.ws + wl.off_h);
  T* ab = reinterpret_cast<T*>(a.ws + wl.off_ab);
  float* o = reinterpret_cast<float*>(a.ws + wl.off_o);
  int* status = device_status_ptr();
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e;

  *stage = "fused projection";
  cudaFuncSetAttribute(tm_proj_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, TP_SMEM);
  const long long ptiles = (P + TILE - 1) / TILE;
  tm_proj_tc_kernel<T><<<(int)(ptiles < sms ? ptiles : sms), TP_THREADS, TP_SMEM, st>>>(a.z, a.mask, a.packed, gout,
                                                                                       ab, P, N, Np, a.B, status);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;

  *stage = "contraction";
  const bool bf16 = a.dtype == DT_BF16;
  if ((e = launch_contract<T, CT_BM>(ab, bf16, a.outgoing != 0, o, N, Np, planes, sms, status, st)) != cudaSuccess)
    return e;

  *stage = "tail";
  const int grid = (int)((P + TILE - 1) / TILE);
  if (a.ln_out && a.tb_next) {
    cudaFuncSetAttribute(tm_tail_tc_kernel<T, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TT_SMEM);
    tm_tail_tc_kernel<T, true, true><<<grid, TT_THREADS, TT_SMEM, st>>>(
        o, a.packed, gout, a.z, a.out, P, N, Np, a.add_residual, a.ln_next_w, a.ln_next_b,
        reinterpret_cast<T*>(a.ln_out), a.tb_next_w, reinterpret_cast<__half*>(a.tb_next), status);
  } else if (a.ln_out) {
    cudaFuncSetAttribute(tm_tail_tc_kernel<T, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TT_SMEM);
    tm_tail_tc_kernel<T, true, false><<<grid, TT_THREADS, TT_SMEM, st>>>(
        o, a.packed, gout, a.z, a.out, P, N, Np, a.add_residual, a.ln_next_w, a.ln_next_b,
        reinterpret_cast<T*>(a.ln_out), nullptr, nullptr, status);
  } else {
    cudaFuncSetAttribute(tm_tail_tc_kernel<T, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TT_SMEM);
    tm_tail_tc_kernel<T, false, false><<<grid, TT_THREADS, TT_SMEM, st>>>(
        o, a.packed, gout, a.z, a.out, P, N, Np, a.add_residual, nullptr, nullptr, nullptr, nullptr, nullptr, status);
  }
  return cudaGetLastError();
}

// fp32 mode: every step in fp32, the three GEMMs as plain cuBLAS fp32 GEMMs (no TF32).
cudaError_t trimul_run32(const TrimulArgs& a, cudaStream_t st, int* blas_status, const char** stage) {
  using T = float;
  const TrimulWorkspace wl = TrimulWorkspace::make(a.B, a.N, a.dtype);
  const long long nn = (long long)a.N * a.N, P = (long long)a.B * nn;
  const float* pf = reinterpret_cast<const float*>(a.packed);
  const T* w1 = reinterpret_cast<const T*>(a.packed + TrimulPacked::w1);
  const T* wpo = reinterpret_cast<const T*>(a.packed + TrimulPacked::p_out);
  T* xn = reinterpret_cast<T*>(a.ws + wl.off_xn);
  T* h = reinterpret_cast<T*>(a.ws + wl.off_h);
  T* ab = reinterpret_cast<T*>(a.ws + wl.off_ab);
  float* y = reinterpret_cast<float*>(a.ws + wl.off_ab);  // after G2 has consumed a and b
  float* o = reinterpret_cast<float*>(a.ws + wl.off_o);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e;
  *stage = "layernorm_in";
  tm_ln_in_kernel<T><<<grid_for(P, 8, sms * 16), 256, 0, st>>>(a.z, pf + TrimulPacked::in_w / 4,
                                                                pf + TrimulPacked::in_b / 4, xn, P);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  int herr = 0;
  cublasHandle_t hb = blas_handle(&herr);
  if (!hb) {
    *blas_status = herr;
    *stage = "cublasCreate";
    return cudaErrorUnknown;
  }
  cublasStatus_t s = cublasSetStream(hb, st);
  if (s == CUBLAS_STATUS_SUCCESS) s = cublasSetWorkspace(hb, a.ws + wl.off_blas, TrimulWorkspace::BLAS_BYTES);
  if (s == CUBLAS_STATUS_SUCCESS) s = cublasSetMathMode(hb, CUBLAS_DEFAULT_MATH);  // fp32 stays fp32 (no TF32)
  const float one = 1.0f, zero = 0.0f;
  // G1, row-major h [P][640] = xn [P][128] . (p_in | g_in | g_out)^T (column-major: h^T = W . xn^T)
  if (s == CUBLAS_STATUS_SUCCESS) {
    *stage = "projection GEMM";
    s = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, TM_W1, (int)P, TM_D, &one, w1, CUDA_R_32F, TM_D, xn, CUDA_R_32F, TM_D,
                     &zero, h, CUDA_R_32F, TM_W1, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  }
  if (s != CUBLAS_STATUS_SUCCESS) {
    *blas_status = (int)s;
    return cudaErrorUnknown;
  }
  *stage = "gate";
  tm_gate_kernel<T><<<(int)((P + TM_GP - 1) / TM_GP), 256, 0, st>>>(h, a.mask, ab, P, nn, a.B);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // G2, per (batch, channel), row-major N x N matrices (column-major views are their transposes):
  //   outgoing o = a . b^T   ->  o^T = b . a^T   (op(b) = T on b^T, op(a^T) = N)
  //   incoming o = a^T . b   ->  o^T = b^T . a   (op(b^T) = N, op(a) = T on a^T)
  *stage = "contraction GEMM";
  const T* am = ab;
  const T* bm = ab + (long long)a.B * TM_D * nn;
  s = cublasGemmStridedBatchedEx(hb, a.outgoing ? CUBLAS_OP_T : CUBLAS_OP_N, a.outgoing ? CUBLAS_OP_N : CUBLAS_OP_T,
                                 a.N, a.N, a.N, &one, bm, CUDA_R_32F, a.N, nn, am, CUDA_R_32F, a.N, nn, &zero, o,
                                 CUDA_R_32F, a.N, nn, a.B * TM_D, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (s != CUBLAS_STATUS_SUCCESS) {
    *blas_status = (int)s;
    return cudaErrorUnknown;
  }
  *stage = "layernorm_out";
  tm_ln_out_kernel<T><<<(int)((P + TM_LP - 1) / TM_LP), 256, 0, st>>>(o, pf + TrimulPacked::out_w / 4,
                                                                        pf + TrimulPacked::out_b / 4, xn, P, nn);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // G3 (row-major y [P][128] = norm_out(o) [P][128] . p_out^T), fp32 out
  *stage = "p_out GEMM";
  s = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, TM_D, (int)P, TM_D, &one, wpo, CUDA_R_32F, TM_D, xn, CUDA_R_32F, TM_D,
                   &zero, y, CUDA_R_32F, TM_D, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (s != CUBLAS_STATUS_SUCCESS) {
    *blas_status = (int)s;
    return cudaErrorUnknown;
  }
  *stage = "output gate";
  tm_out_kernel<T><<<grid_for(P * 32, 256, sms * 16), 256, 0, st>>>(a.z, y, h + 4 * TM_D, TM_W1, a.out, P * 32,
                                                                     a.add_residual);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_trimul_pack(const float* in_w, const float* in_b, const float* p_in, const float* g_in,
                               const float* out_w, const float* out_b, const float* p_out, const float* g_out,
                               int dtype, unsigned char* packed, cudaStream_t st) {
  if (dtype == DT_BF16)
    tm_pack_kernel<__nv_bfloat16><<<160, 256, 0, st>>>(in_w, in_b, p_in, g_in, out_w, out_b, p_out, g_out, packed, 1);
  else
    tm_pack_kernel<__half><<<160, 256, 0, st>>>(in_w, in_b, p_in, g_in, out_w, out_b, p_out, g_out, packed,
                                                dtype == DT_F16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_trimul(const TrimulArgs& a, cudaStream_t st, int* blas_status, const char** stage) {
  *blas_status = 0;
  if (a.dtype == DT_F32) return trimul_run32(a, st, blas_status, stage);
  if (a.dtype == DT_BF16) return trimul_run16<__nv_bfloat16>(a, st, stage);
  return trimul_run16<__half>(a, st, stage);
}

}  // namespace triattn
