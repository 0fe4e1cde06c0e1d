// fp32 path of the triangle-attention layer (SIMT FFMA; the tensor cores have no fp32 mode that
// meets the reference's fp32 tolerance), plus the dtype-independent helpers: weight packing and
// the mask-bias preparation.
//
// fp32 arithmetic follows the reference's fp32 ops path
// (boltz_mlx/layers/triangular_attention/attention.py:47-93):
//   xn = LN(x) (two-pass fp32 statistics, eps 1e-5, kernels.py:438-464)
//   q = (xn Wq^T) * C^-1/2, k, v, g = xn W^T (+ g bias); tri_bias = xn Wb^T
//   a = q k^T + (tri_bias + inf*(mask-1))   -- the bias is summed first, as attention.py:86 does
//   o = softmax(a) v ;  core = o * sigmoid(g) ;  y = core Wo^T (+ z)
#include "sm100.cuh"
#include "triattn_internal.cuh"

namespace triattn {

// ------------------------------------------------------------------------------------------------
// weight packing
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void pack_weights_kernel(const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                                    const float* __restrict__ w_q, const float* __restrict__ w_k,
                                    const float* __restrict__ w_v, const float* __restrict__ w_g,
                                    const float* __restrict__ g_bias, const float* __restrict__ w_b,
                                    const float* __restrict__ w_o, unsigned char* __restrict__ packed,
                                    int with_images) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nthreads = gridDim.x * blockDim.x;
  float* f = reinterpret_cast<float*>(packed);
  for (int i = tid; i < C_IN; i += nthreads) {
    f[PackedLayout::ln_w / 4 + i] = ln_w[i];
    f[PackedLayout::ln_b / 4 + i] = ln_b[i];
    f[PackedLayout::g_b / 4 + i] = g_bias ? g_bias[i] : 0.0f;
  }
  for (int i = tid; i < HEADS * C_IN; i += nthreads) f[PackedLayout::w_b / 4 + i] = w_b[i];
  for (int i = tid; i < NPROJ * C_IN; i += nthreads) {
    const int n = i / C_IN, k = i % C_IN;
    const float* src = n < HC ? w_q : n < 2 * HC ? w_k : n < 3 * HC ? w_v : w_g;
    const float v = src[(n % HC) * C_IN + k];
    f[PackedLayout::w_qkvg / 4 + i] = v;
    if (with_images) {
      T* img = reinterpret_cast<T*>(packed + PackedLayout::img_qkvg);
      img[img_off(n, k, C_IN) / 2] = T(v);
    }
  }
  for (int i = tid; i < C_IN * HC; i += nthreads) {
    const int n = i / HC, k = i % HC;
    const float v = w_o[i];
    f[PackedLayout::w_o / 4 + i] = v;
    if (with_images) {
      T* img = reinterpret_cast<T*>(packed + PackedLayout::img_o);
      img[img_off(n, k, HC) / 2] = T(v);
    }
  }
}

cudaError_t launch_pack_weights(const float* ln_w, const float* ln_b, const float* w_q, const float* w_k,
                                const float* w_v, const float* w_g, const float* g_bias, const float* w_b,
                                const float* w_o, int dtype, unsigned char* packed, cudaStream_t st) {
  if (dtype == DT_F16)
    pack_weights_kernel<__half><<<128, 256, 0, st>>>(ln_w, ln_b, w_q, w_k, w_v, w_g, g_bias, w_b, w_o, packed, 1);
  else if (dtype == DT_BF16)
    pack_weights_kernel<__nv_bfloat16>
        <<<128, 256, 0, st>>>(ln_w, ln_b, w_q, w_k, w_v, w_g, g_bias, w_b, w_o, packed, 1);
  else
    pack_weights_kernel<__half><<<128, 256, 0, st>>>(ln_w, ln_b, w_q, w_k, w_v, w_g, g_bias, w_b, w_o, packed, 0);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// mask bias: mb[b][a - row_begin][k] = inf * (mask_att[b][a][k] - 1)  (x log2e on the 16-bit path),
// keys k >= N padded (-1e30 on the 16-bit path, which masks them out of every row).
// Reference: attention.py:85 (mask_bias), kernels_nax.py:496-503 (log2-domain, padded keys).
// ------------------------------------------------------------------------------------------------
__global__ void mask_prep_kernel(const float* __restrict__ mask, View mv, int B, int N, int Np, int row_begin,
                                 int R, float inf, int log2_domain, float* __restrict__ mb) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  const int al = blockIdx.y;
  const int b = blockIdx.z;
  if (k >= Np) return;
  const int a = row_begin + al;
  float v;
  if (k < N) {
    const float m = mask ? mask[b * mv.s_batch + (long long)(a - mv.row0) * mv.s_row + view_col(mv, k)] : 1.0f;
    v = inf * (m - 1.0f);
    if (log2_domain) v *= LOG2E;
  } else {
    v = log2_domain ? -1e30f : 0.0f;
  }
  mb[((size_t)b * R + al) * Np + k] = v;
}

cudaError_t launch_mask_prep(const LayerArgs& a, int dtype, cudaStream_t st) {
  if (dtype != DT_F32) return launch_mask_prep_tc(a, st);
  const int R = a.row_end - a.row_begin;
  float* mb = reinterpret_cast<float*>(a.ws + a.wl.off_mb);
  dim3 grid((a.wl.Np + 255) / 256, R, a.B);
  mask_prep_kernel<<<grid, 256, 0, st>>>(a.mask, a.mv, a.B, a.N, a.wl.Np, a.row_begin, R, a.inf, dtype != DT_F32, mb);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// fp32 LayerNorm + projection: 64 pairs (a, c0..c0+63) per CTA, 256 threads.
// ------------------------------------------------------------------------------------------------
namespace {
constexpr int F_ROWS = 64;
constexpr int F_LD = 68;  // padded leading dimension of the transposed smem tiles (float4-aligned)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
}  // namespace

__global__ void __launch_bounds__(256) ln_proj_f32_kernel(LayerArgs args) {
  extern __shared__ __align__(16) float smem_f[];
  float* xT = smem_f;                  // [128][F_LD]
  float* wT = smem_f + C_IN * F_LD;    // [128][F_LD]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * F_ROWS;
  const int al = blockIdx.y, a = args.row_begin + al;
  const int b = blockIdx.z;
  const int N = args.N, R = args.row_end - args.row_begin;
  const float* P = reinterpret_cast<const float*>(args.packed);

  // ---- LayerNorm (warp per row; lane owns channels 4*lane..4*lane+3) ----
  const float4 lw = reinterpret_cast<const float4*>(P + PackedLayout::ln_w / 4)[lane];
  const float4 lb = reinterpret_cast<const float4*>(P + PackedLayout::ln_b / 4)[lane];
  for (int r = warp; r < F_ROWS; r += 8) {
    const int c = c0 + r;
    float4 xn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < N) {
      const float* x = args.z + b * args.zv.s_batch + (long long)(a - args.zv.row0) * args.zv.s_row +
                       view_col(args.zv, c);
      const float4 v = reinterpret_cast<const float4*>(x)[lane];
      const float mean = warp_sum(v.x + v.y + v.z + v.w) * (1.0f / C_IN);
      const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
      const float var = warp_sum(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3) * (1.0f / C_IN);
      const float rstd = 1.0f / sqrtf(var + LN_EPS);
      xn = make_float4(d0 * rstd * lw.x + lb.x, d1 * rstd * lw.y + lb.y, d2 * rstd * lw.z + lb.z,
                       d3 * rstd * lw.w + lb.w);
    }
    xT[(4 * lane + 0) * F_LD + r] = xn.x;
    xT[(4 * lane + 1) * F_LD + r] = xn.y;
    xT[(4 * lane + 2) * F_LD + r] = xn.z;
    xT[(4 * lane + 3) * F_LD + r] = xn.w;
  }

  const int ty = tid >> 4, tx = tid & 15;  // rows ty*4.., cols tx*4..
  const float scale = rsqrtf((float)C_HEAD);
  const int Np = args.wl.Np;
  float* q = reinterpret_cast<float*>(args.ws + args.wl.off_q);
  float* k = reinterpret_cast<float*>(args.ws + args.wl.off_k);
  float* v = reinterpret_cast<float*>(args.ws + args.wl.off_v);
  float* g = reinterpret_cast<float*>(args.ws + args.wl.off_g);
  float* bias = reinterpret_cast<float*>(args.ws + args.wl.off_bias);

  for (int cc = 0; cc < 9; ++cc) {  // 9 chunks of 64 output columns cover q|k|v|g (512) + tri bias (4)
    const int o0 = cc * 64;
    __syncthreads();
    for (int idx = tid; idx < 64 * C_IN; idx += 256) {
      const int j = idx / C_IN, kk = idx % C_IN, o = o0 + j;
      float w = 0.f;
      if (o < NPROJ) w = P[PackedLayout::w_qkvg / 4 + o * C_IN + kk];
      else if (o < NPROJ + HEADS) w = P[PackedLayout::w_b / 4 + (o - NPROJ) * C_IN + kk];
      wT[kk * F_LD + j] = w;
    }
    __syncthreads();
    float acc[4][4] = {};
#pragma unroll 8
    for (int kk = 0; kk < C_IN; ++kk) {
      const float4 xv = *reinterpret_cast<const float4*>(xT + kk * F_LD + ty * 4);
      const float4 wv = *reinterpret_cast<const float4*>(wT + kk * F_LD + tx * 4);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + ty * 4 + i;
      if (c >= N) continue;
      const size_t prow = (((size_t)b * R + al) * N + c) * C_IN;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int o = o0 + tx * 4 + j;
        const float val = acc[i][j];
        if (o < HC) q[prow + o] = val * scale;
        else if (o < 2 * HC) k[prow + o - HC] = val;
        else if (o < 3 * HC) v[prow + o - 2 * HC] = val;
        else if (o < 4 * HC) g[prow + o - 3 * HC] = val + P[PackedLayout::g_b / 4 + (o - 3 * HC)];
        else if (o < NPROJ + HEADS)
          bias[(((size_t)a * args.B + b) * HEADS + (o - NPROJ)) * Np + c] = val;
      }
    }
  }
}

cudaError_t launch_ln_proj_f32(const LayerArgs& a, cudaStream_t st) {
  const int R = a.row_end - a.row_begin;
  const size_t smem = 2 * C_IN * F_LD * sizeof(float);
  cudaFuncSetAttribute(ln_proj_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((a.N + F_ROWS - 1) / F_ROWS, R, a.B);
  ln_proj_f32_kernel<<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// fp32 flash core: one thread per query j; 64 queries of one (b, row a, head h) per CTA.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(64) core_f32_kernel(LayerArgs args) {
  __shared__ __align__(16) float Ks[64][C_HEAD];
  __shared__ __align__(16) float Vs[64][C_HEAD];
  __shared__ float Ms[64];
  const int tid = threadIdx.x;
  const int j = blockIdx.x * 64 + tid;
  const int al = blockIdx.y;
  const int b = blockIdx.z / HEADS, h = blockIdx.z % HEADS;
  const int N = args.N, R = args.row_end - args.row_begin, Np = args.wl.Np;
  const bool valid = j < N;
  const int jc = valid ? j : N - 1;
  const float* q = reinterpret_cast<const float*>(args.ws + args.wl.off_q);
  const float* kb = reinterpret_cast<const float*>(args.ws + args.wl.off_k);
  const float* vb = reinterpret_cast<const float*>(args.ws + args.wl.off_v);
  const float* g = reinterpret_cast<const float*>(args.ws + args.wl.off_g);
  const float* bias = reinterpret_cast<const float*>(args.ws + args.wl.off_bias);
  const float* mb = reinterpret_cast<const float*>(args.ws + args.wl.off_mb) + ((size_t)b * R + al) * Np;
  float* core = reinterpret_cast<float*>(args.ws + args.wl.off_core);

  const size_t rowbase = ((size_t)b * R + al) * N;  // pair (b, a, 0)
  float qv[C_HEAD], o[C_HEAD];
#pragma unroll
  for (int d = 0; d < C_HEAD; d += 4) {
    const float4 t = *reinterpret_cast<const float4*>(q + (rowbase + jc) * C_IN + h * C_HEAD + d);
    qv[d] = t.x; qv[d + 1] = t.y; qv[d + 2] = t.z; qv[d + 3] = t.w;
    o[d] = o[d + 1] = o[d + 2] = o[d + 3] = 0.f;
  }
  const float* tb = bias + (((size_t)jc * args.B + b) * HEADS + h) * Np;
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < N; k0 += 64) {
    const int nk = min(64, N - k0);
    __syncthreads();
    if (tid < nk) {
      const float* ks = kb + (rowbase + k0 + tid) * C_IN + h * C_HEAD;
      const float* vs = vb + (rowbase + k0 + tid) * C_IN + h * C_HEAD;
#pragma unroll
      for (int d = 0; d < C_HEAD; d += 4) {
        *reinterpret_cast<float4*>(&Ks[tid][d]) = *reinterpret_cast<const float4*>(ks + d);
        *reinterpret_cast<float4*>(&Vs[tid][d]) = *reinterpret_cast<const float4*>(vs + d);
      }
      Ms[tid] = mb[k0 + tid];
    }
    __syncthreads();
    float s[64];
    float tmax = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < 64; ++kk) {
      if (kk < nk) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < C_HEAD; ++d) dot = fmaf(qv[d], Ks[kk][d], dot);
        const float t = tb[k0 + kk] + Ms[kk];  // tri_bias + mask_bias (attention.py:86)
        s[kk] = dot + t;
        tmax = fmaxf(tmax, s[kk]);
      } else {
        s[kk] = -INFINITY;
      }
    }
    const float m_new = fmaxf(m, tmax);
    const float corr = expf(m - m_new);
    l *= corr;
#pragma unroll
    for (int d = 0; d < C_HEAD; ++d) o[d] *= corr;
#pragma unroll
    for (int kk = 0; kk < 64; ++kk) {
      if (kk < nk) {
        const float p = expf(s[kk] - m_new);
        l += p;
#pragma unroll
        for (int d = 0; d < C_HEAD; ++d) o[d] = fmaf(p, Vs[kk][d], o[d]);
      }
    }
    m = m_new;
  }
  if (!valid) return;
  const float inv_l = 1.0f / l;
  const float* gr = g + (rowbase + j) * C_IN + h * C_HEAD;
  float* out = core + (rowbase + j) * C_IN + h * C_HEAD;
#pragma unroll
  for (int d = 0; d < C_HEAD; d += 4) {
    const float4 gv = *reinterpret_cast<const float4*>(gr + d);
    float4 r;
    r.x = (o[d] * inv_l) * (1.0f / (1.0f + expf(-gv.x)));
    r.y = (o[d + 1] * inv_l) * (1.0f / (1.0f + expf(-gv.y)));
    r.z = (o[d + 2] * inv_l) * (1.0f / (1.0f + expf(-gv.z)));
    r.w = (o[d + 3] * inv_l) * (1.0f / (1.0f + expf(-gv.w)));
    *reinterpret_cast<float4*>(out + d) = r;
  }
}

cudaError_t launch_core_f32(const LayerArgs& a, cudaStream_t st) {
  const int R = a.row_end - a.row_begin;
  dim3 grid((a.N + 63) / 64, R, a.B * HEADS);
  core_f32_kernel<<<grid, 64, 0, st>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// fp32 output projection (+ residual): 64 pairs per CTA, 256 threads, written in z's orientation.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) out_proj_f32_kernel(LayerArgs args) {
  extern __shared__ __align__(16) float smem_f[];
  float* cT = smem_f;               // [128][F_LD]
  float* wT = smem_f + HC * F_LD;   // [128][F_LD]
  const int tid = threadIdx.x;
  const int c0 = blockIdx.x * F_ROWS;
  const int al = blockIdx.y, a = args.row_begin + al;
  const int b = blockIdx.z;
  const int N = args.N, R = args.row_end - args.row_begin;
  const float* P = reinterpret_cast<const float*>(args.packed);
  const float* core = reinterpret_cast<const float*>(args.ws + args.wl.off_core);
  for (int idx = tid; idx < F_ROWS * HC; idx += 256) {
    const int r = idx / HC, kk = idx % HC, c = c0 + r;
    cT[kk * F_LD + r] = c < N ? core[(((size_t)b * R + al) * N + c) * HC + kk] : 0.f;
  }
  const int ty = tid >> 4, tx = tid & 15;
  for (int cc = 0; cc < 2; ++cc) {
    const int o0 = cc * 64;
    __syncthreads();
    for (int idx = tid; idx < 64 * HC; idx += 256) {
      const int j = idx / HC, kk = idx % HC;
      wT[kk * F_LD + j] = P[PackedLayout::w_o / 4 + (o0 + j) * HC + kk];
    }
    __syncthreads();
    float acc[4][4] = {};
#pragma unroll 8
    for (int kk = 0; kk < HC; ++kk) {
      const float4 xv = *reinterpret_cast<const float4*>(cT + kk * F_LD + ty * 4);
      const float4 wv = *reinterpret_cast<const float4*>(wT + kk * F_LD + tx * 4);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + ty * 4 + i;
      if (c >= N) continue;
      const long long off = b * args.ov.s_batch + (long long)(a - args.ov.row0) * args.ov.s_row +
                            view_col(args.ov, c) + o0 + tx * 4;
      float4 r = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      if (args.add_residual) {
        const long long zoff = b * args.zv.s_batch + (long long)(a - args.zv.row0) * args.zv.s_row +
                               view_col(args.zv, c) + o0 + tx * 4;
        const float4 zz = *reinterpret_cast<const float4*>(args.z + zoff);
        r.x += zz.x; r.y += zz.y; r.z += zz.z; r.w += zz.w;
      }
      *reinterpret_cast<float4*>(args.out + off) = r;
    }
  }
  // peer stores (output blocks in other GPUs' memory): performed system-wide before the kernel ends,
  // ahead of the cross-GPU barrier that publishes them
  if (args.ov.tab) __threadfence_system();
}

cudaError_t launch_out_proj_f32(const LayerArgs& a, cudaStream_t st) {
  const int R = a.row_end - a.row_begin;
  const size_t smem = 2 * HC * F_LD * sizeof(float);
  cudaFuncSetAttribute(out_proj_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((a.N + F_ROWS - 1) / F_ROWS, R, a.B);
  out_proj_f32_kernel<<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace triattn
