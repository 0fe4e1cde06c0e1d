// Triangle multiplication, outgoing and incoming edges (boltz_mlx/layers/triangular_mult.py:10-178),
// forward only, on a B200:
//
//   K1  LayerNorm-in, one warp per pair (two-pass fp32 statistics)      z fp32 -> xn [P][128]
//   G1  cuBLAS GEMM   h = xn . [p_in | g_in | g_out]^T                  -> h [P][640]
//   K2  gate + mask, transposed through shared memory to channel-major  -> a, b [B][128][N][N]
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
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <mutex>

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
                                                     const T* __restrict__ h, float* out, long long n4,
                                                     int add_residual) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const long long p = i >> 5, c = (i & 31) * 4;  // 32 float4 per pair
    const float4 yv = __ldcs(reinterpret_cast<const float4*>(y) + i);
    const float4 g = Ew<T>::ld4(h + p * TM_W1 + 4 * TM_D + c);
    float4 r = make_float4(yv.x * tm_sigmoid(g.x), yv.y * tm_sigmoid(g.y), yv.z * tm_sigmoid(g.z),
                           yv.w * tm_sigmoid(g.w));
    if (add_residual) {
      const float4 zv = reinterpret_cast<const float4*>(z)[i];  // out may alias z: read before write
      r.x += zv.x; r.y += zv.y; r.z += zv.z; r.w += zv.w;
    }
    reinterpret_cast<float4*>(out)[i] = r;
  }
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
    if (with16) reinterpret_cast<T*>(packed + TrimulPacked::w1_16)[i] = static_cast<T>(v);
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

template <typename T>
cudaDataType_t cuda_type();
template <>
cudaDataType_t cuda_type<float>() { return CUDA_R_32F; }
template <>
cudaDataType_t cuda_type<__half>() { return CUDA_R_16F; }
template <>
cudaDataType_t cuda_type<__nv_bfloat16>() { return CUDA_R_16BF; }

int grid_for(long long work, int per_block, int cap) {
  const long long g = (work + per_block - 1) / per_block;
  return (int)(g < cap ? (g < 1 ? 1 : g) : cap);
}

template <typename T>
cudaError_t trimul_run(const TrimulArgs& a, cudaStream_t st, int* blas_status, const char** stage) {
  const TrimulWorkspace wl = TrimulWorkspace::make(a.B, a.N, a.dtype);
  const long long nn = (long long)a.N * a.N, P = (long long)a.B * nn;
  const float* pf = reinterpret_cast<const float*>(a.packed);
  const T* w1 = reinterpret_cast<const T*>(a.packed + (sizeof(T) == 4 ? TrimulPacked::w1 : TrimulPacked::w1_16));
  const T* wpo = reinterpret_cast<const T*>(a.packed + (sizeof(T) == 4 ? TrimulPacked::p_out : TrimulPacked::p_out_16));
  T* xn = reinterpret_cast<T*>(a.ws + wl.off_xn);
  T* h = reinterpret_cast<T*>(a.ws + wl.off_h);
  T* ab = reinterpret_cast<T*>(a.ws + wl.off_ab);
  float* y = reinterpret_cast<float*>(a.ws + wl.off_ab);  // after G2 has consumed a and b
  float* o = reinterpret_cast<float*>(a.ws + wl.off_o);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);

  *stage = "layernorm_in";
  tm_ln_in_kernel<T><<<grid_for(P, 8, sms * 16), 256, 0, st>>>(a.z, pf + TrimulPacked::in_w / 4,
                                                                pf + TrimulPacked::in_b / 4, xn, P);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

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
  const cudaDataType_t tt = cuda_type<T>();
  const float one = 1.0f, zero = 0.0f;
  // G1 (row-major h [P][640] = xn [P][128] . W1^T; column-major: h^T = W1 . xn^T)
  if (s == CUBLAS_STATUS_SUCCESS) {
    *stage = "projection GEMM";
    s = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, TM_W1, (int)P, TM_D, &one, w1, tt, TM_D, xn, tt, TM_D, &zero, h, tt,
                     TM_W1, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
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
                                 a.N, a.N, a.N, &one, bm, tt, a.N, nn, am, tt, a.N, nn, &zero, o, CUDA_R_32F, a.N, nn,
                                 a.B * TM_D, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
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
  s = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, TM_D, (int)P, TM_D, &one, wpo, tt, TM_D, xn, tt, TM_D, &zero, y,
                   CUDA_R_32F, TM_D, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (s != CUBLAS_STATUS_SUCCESS) {
    *blas_status = (int)s;
    return cudaErrorUnknown;
  }
  *stage = "output gate";
  tm_out_kernel<T><<<grid_for(P * 32, 256, sms * 16), 256, 0, st>>>(a.z, y, h, a.out, P * 32, a.add_residual);
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
  if (a.dtype == DT_F32) return trimul_run<float>(a, st, blas_status, stage);
  if (a.dtype == DT_BF16) return trimul_run<__nv_bfloat16>(a, st, blas_status, stage);
  return trimul_run<__half>(a, st, blas_status, stage);
}

}  // namespace triattn
