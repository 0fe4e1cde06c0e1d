// 16-bit (fp16 / bf16) path of the triangle-attention layer on the sm_100a tensor cores (tcgen05,
// accumulators in TMEM), fp32 accumulation / softmax statistics / residual.
//
// Data flow of one layer (attention orientation x[a][c]; ending node: x[a][c] = z[c][a], read in
// place through strides):
//   ln_proj_tc : z rows -> LN (fp32 stats) -> xn 16-bit operand image in smem -> UMMA with the
//                W_qkvg image (512 x 128) -> q, k, v operand images (8 KB per 128-position tile and
//                head), g (row-major 16-bit); tri bias (fp32 SIMT dot from fp32 xn, x log2e).
//   core_tc    : per (b, row a, head h, 128-query tile): S = Q K^T (UMMA, SS) in TMEM ->
//                log2-domain logits fma(S, C^-1/2 log2e, mask bias) + tri bias, online softmax
//                (fp32) -> P (16-bit) stored to TMEM -> O_part = P V (UMMA, A from TMEM) ->
//                accumulated in registers; epilogue o / l * sigmoid(g) -> core operand image.
//   out_proj_tc: y = core W_o^T (UMMA) -> (+ z) -> out, written in z's orientation.
//
// Every operand image uses the no-swizzle K-major core-matrix layout of sm100.cuh (img_off), so a
// whole tile moves with ONE 1-D bulk copy and no tensor map.  All waits are bounded.
//
// Reference counterparts (jackryan225/boltz-mlx): kernels.py:438-464 (LN), kernels_nax3.py:538-677
// (q|k|v|g projection), kernels_nax.py:323-469 (16-bit flash tri-attention with log2-domain
// logits, exp2 online softmax, sigmoid gate), kernels_nax3.py:176-198 (linear_o epilogue).
#include "sm100.cuh"
#include "triattn_internal.cuh"

namespace triattn {

namespace {
__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
}  // namespace

// =================================================================================================
// LN + q|k|v|g projection (+ tri bias).  CTA = 128 pairs (a, c0..c0+127) of one attention row,
// 256 threads (8 warps).  TMEM: 512 columns = the full 128 x 512 fp32 accumulator.
// =================================================================================================
constexpr int LP_W_BYTES = NPROJ * C_IN * 2;  // 131072
constexpr int LP_A_BYTES = TILE * C_IN * 2;   // 32768
constexpr int LP_SMEM = LP_W_BYTES + LP_A_BYTES + HEADS * TILE * 4 + 64;

template <typename T>
__global__ void __launch_bounds__(256, 1) ln_proj_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sW = smem;
  unsigned char* sA = smem + LP_W_BYTES;
  float* sBias = reinterpret_cast<float*>(smem + LP_W_BYTES + LP_A_BYTES);  // [4][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LP_W_BYTES + LP_A_BYTES + HEADS * TILE * 4);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  uint64_t* bar_w = bars;
  uint64_t* bar_mma = bars + 1;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ct = blockIdx.x, c0 = ct * TILE;
  const int al = blockIdx.y, a = args.row_begin + al;
  const int b = blockIdx.z;
  const int N = args.N, R = args.row_end - args.row_begin, Np = args.wl.Np, NT = args.wl.NT;
  const float* P = reinterpret_cast<const float*>(args.packed);
  int* status = args.status;

  if (tid == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_w, LP_W_BYTES);
    bulk_g2s(sW, args.packed + PackedLayout::img_qkvg, LP_W_BYTES, bar_w);
  }

  // ---- LayerNorm: warp w handles rows 16w..16w+15; lane owns channels 4*lane..4*lane+3 ----
  const float4 lw = reinterpret_cast<const float4*>(P + PackedLayout::ln_w / 4)[lane];
  const float4 lb = reinterpret_cast<const float4*>(P + PackedLayout::ln_b / 4)[lane];
  float4 wb[HEADS];
#pragma unroll
  for (int hh = 0; hh < HEADS; ++hh) wb[hh] = reinterpret_cast<const float4*>(P + PackedLayout::w_b / 4 + hh * C_IN)[lane];
  float4 xv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = c0 + warp * 16 + i;
    xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < N) {
      const float* x = args.z + b * args.zv.s_batch + (long long)(a - args.zv.row0) * args.zv.s_row +
                       (long long)c * args.zv.s_col;
      xv[i] = __ldg(reinterpret_cast<const float4*>(x) + lane);
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int r = warp * 16 + i;
    const float4 v = xv[i];
    const float mean = warp_sum32(v.x + v.y + v.z + v.w) * (1.0f / C_IN);
    const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
    const float var = warp_sum32(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3) * (1.0f / C_IN);
    const float rstd = 1.0f / sqrtf(var + LN_EPS);
    const float n0 = d0 * rstd * lw.x + lb.x, n1 = d1 * rstd * lw.y + lb.y;
    const float n2 = d2 * rstd * lw.z + lb.z, n3 = d3 * rstd * lw.w + lb.w;
    uint2 pk;
    pk.x = H16<T>::pack(n0, n1);
    pk.y = H16<T>::pack(n2, n3);
    *reinterpret_cast<uint2*>(sA + img_off(r, 4 * lane, C_IN)) = pk;
    float tbv[HEADS];
#pragma unroll
    for (int hh = 0; hh < HEADS; ++hh)
      tbv[hh] = warp_sum32(n0 * wb[hh].x + n1 * wb[hh].y + n2 * wb[hh].z + n3 * wb[hh].w);
    if (lane == 0) {
#pragma unroll
      for (int hh = 0; hh < HEADS; ++hh) sBias[hh * TILE + r] = tbv[hh];
    }
  }
  fence_proxy_async_smem();
  __syncthreads();

  // ---- tri bias rows: bias[a][b][h][c] (log2 domain; padded columns 0) ----
  {
    float* bias = reinterpret_cast<float*>(args.ws + args.wl.off_bias);
    for (int idx = tid; idx < HEADS * TILE; idx += 256) {
      const int hh = idx / TILE, r = idx % TILE, c = c0 + r;
      bias[(((size_t)a * args.B + b) * HEADS + hh) * Np + c] = c < N ? sBias[idx] * LOG2E : 0.0f;
    }
  }

  // ---- MMA: D[128 x 512] = xn[128 x 128] * W_qkvg[512 x 128]^T, two N=256 halves ----
  if (tid == 0) {
    mbar_wait(bar_w, 0, status, DEV_TIMEOUT_TMA);
    tc_fence_after();
    constexpr uint32_t idesc = make_idesc_f16(128, 256, H16<T>::is_bf16, 0, 0);
#pragma unroll
    for (int ks = 0; ks < C_IN / 16; ++ks) {
      const uint64_t ad = smem_desc_noswizzle(smem_u32(sA) + ks * 256, 128, 16 * C_IN);
#pragma unroll
      for (int nh = 0; nh < 2; ++nh) {
        const uint64_t bd = smem_desc_noswizzle(smem_u32(sW) + nh * 65536 + ks * 256, 128, 16 * C_IN);
        umma_ss(tbase + nh * 256, ad, bd, idesc, ks > 0 ? 1u : 0u);
      }
    }
    umma_commit(bar_mma);
  }
  __syncwarp();
  mbar_wait(bar_mma, 0, status, DEV_TIMEOUT_MMA);
  __syncwarp();
  tc_fence_after();

  // ---- epilogue: warp w reads lanes 32*(w%4).., column half w/4 (q|k or v|g) ----
  const int quad = warp & 3, half = warp >> 2;
  const int r = quad * 32 + lane, c = c0 + r;
  const bool valid = c < N;
#pragma unroll 1
  for (int t = 0; t < 2; ++t) {
    const int tt = half * 2 + t;  // 0 q, 1 k, 2 v, 3 g
#pragma unroll 1
    for (int hh = 0; hh < HEADS; ++hh) {
      uint32_t acc[32];
      tmem_ld32(tmem_addr(tbase, quad * 32, tt * 128 + hh * 32), acc);
      tmem_ld_wait();
      if (tt < 3) {
        const size_t off = (tt == 0 ? args.wl.off_q : tt == 1 ? args.wl.off_k : args.wl.off_v) +
                           ((((size_t)b * R + al) * HEADS + hh) * NT + ct) * 8192;
        unsigned char* img = args.ws + off;
#pragma unroll
        for (int d = 0; d < C_HEAD; d += 8) {
          uint4 pk = make_uint4(0u, 0u, 0u, 0u);
          if (valid) {
            pk.x = H16<T>::pack(__uint_as_float(acc[d + 0]), __uint_as_float(acc[d + 1]));
            pk.y = H16<T>::pack(__uint_as_float(acc[d + 2]), __uint_as_float(acc[d + 3]));
            pk.z = H16<T>::pack(__uint_as_float(acc[d + 4]), __uint_as_float(acc[d + 5]));
            pk.w = H16<T>::pack(__uint_as_float(acc[d + 6]), __uint_as_float(acc[d + 7]));
          }
          *reinterpret_cast<uint4*>(img + img_off(r, d, C_HEAD)) = pk;
        }
      } else if (valid) {
        const float* gb = P + PackedLayout::g_b / 4 + hh * C_HEAD;
        T* g = reinterpret_cast<T*>(args.ws + args.wl.off_g) + (((size_t)b * R + al) * N + c) * C_IN + hh * C_HEAD;
#pragma unroll
        for (int d = 0; d < C_HEAD; d += 8) {
          uint4 pk;
          pk.x = H16<T>::pack(__uint_as_float(acc[d + 0]) + gb[d + 0], __uint_as_float(acc[d + 1]) + gb[d + 1]);
          pk.y = H16<T>::pack(__uint_as_float(acc[d + 2]) + gb[d + 2], __uint_as_float(acc[d + 3]) + gb[d + 3]);
          pk.z = H16<T>::pack(__uint_as_float(acc[d + 4]) + gb[d + 4], __uint_as_float(acc[d + 5]) + gb[d + 5]);
          pk.w = H16<T>::pack(__uint_as_float(acc[d + 6]) + gb[d + 6], __uint_as_float(acc[d + 7]) + gb[d + 7]);
          *reinterpret_cast<uint4*>(g + d) = pk;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

template <typename T>
static cudaError_t ln_proj_tc_launch(const LayerArgs& a, cudaStream_t st) {
  cudaFuncSetAttribute(ln_proj_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, LP_SMEM);
  const int R = a.row_end - a.row_begin;
  dim3 grid(a.wl.NT, R, a.B);
  ln_proj_tc_kernel<T><<<grid, 256, LP_SMEM, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ln_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  return dtype == DT_BF16 ? ln_proj_tc_launch<__nv_bfloat16>(a, st) : ln_proj_tc_launch<__half>(a, st);
}

// =================================================================================================
// Flash core.  CTA = 128 queries of one (b, attention row a, head h); 128 threads, thread t owns
// query qt*128 + t = TMEM lane t.  TMEM: S / P at columns [0,128), O partial at [128,160).
// =================================================================================================
constexpr int CORE_SMEM_FIXED = 8192 * 5 + 128;  // Q, K[2], V[2], barriers + TMEM slot

template <typename T>
__global__ void __launch_bounds__(128) core_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sQ = smem;
  unsigned char* sK[2] = {smem + 8192, smem + 16384};
  unsigned char* sV[2] = {smem + 24576, smem + 32768};
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 40960);  // q, kv0, kv1, mma
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 40960 + 64);
  float* sMB = reinterpret_cast<float*>(smem + CORE_SMEM_FIXED);  // mask-bias row [Np]
  uint64_t* bar_q = bars;
  uint64_t* bar_kv = bars + 1;
  uint64_t* bar_mma = bars + 3;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int qt = blockIdx.x;
  const int al = blockIdx.y;
  const int b = blockIdx.z / HEADS, h = blockIdx.z % HEADS;
  const int N = args.N, R = args.row_end - args.row_begin, Np = args.wl.Np, NT = args.wl.NT;
  const int q = qt * TILE + tid;
  const bool valid = q < N;
  const int qc = valid ? q : N - 1;
  int* status = args.status;

  const size_t head_tile0 = (((size_t)b * R + al) * HEADS + h) * NT;
  const unsigned char* qimg = args.ws + args.wl.off_q + (head_tile0 + qt) * 8192;
  const unsigned char* kimg = args.ws + args.wl.off_k + head_tile0 * 8192;
  const unsigned char* vimg = args.ws + args.wl.off_v + head_tile0 * 8192;
  const float* mbrow = reinterpret_cast<const float*>(args.ws + args.wl.off_mb) + ((size_t)b * R + al) * Np;
  const float* tb = reinterpret_cast<const float*>(args.ws + args.wl.off_bias) +
                    (((size_t)qc * args.B + b) * HEADS + h) * Np;

  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_kv + 0, 1);
    mbar_init(bar_kv + 1, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tS = tbase, tO = tbase + 128;

  if (tid == 0) {
    mbar_arrive_expect_tx(bar_q, 8192 + Np * 4);
    bulk_g2s(sQ, qimg, 8192, bar_q);
    bulk_g2s(sMB, mbrow, Np * 4, bar_q);
    for (int s = 0; s < 2 && s < NT; ++s) {
      mbar_arrive_expect_tx(bar_kv + s, 16384);
      bulk_g2s(sK[s], kimg + (size_t)s * 8192, 8192, bar_kv + s);
      bulk_g2s(sV[s], vimg + (size_t)s * 8192, 8192, bar_kv + s);
    }
  }

  constexpr uint32_t idS = make_idesc_f16(128, 128, H16<T>::is_bf16, 0, 0);
  constexpr uint32_t idO = make_idesc_f16(128, C_HEAD, H16<T>::is_bf16, 0, 1);
  const float c_l2 = 0.17677669529663687f * LOG2E;  // C^-1/2 * log2(e)
  float m = -INFINITY, l = 0.f;
  float o[C_HEAD];
#pragma unroll
  for (int d = 0; d < C_HEAD; ++d) o[d] = 0.f;
  uint32_t mph = 0;
  mbar_wait(bar_q, 0, status, DEV_TIMEOUT_TMA);
  __syncwarp();

  for (int kt = 0; kt < NT; ++kt) {
    const int s = kt & 1;
    if (tid == 0) {
      mbar_wait(bar_kv + s, (kt >> 1) & 1, status, DEV_TIMEOUT_TMA);
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < C_HEAD / 16; ++ks) {
        const uint64_t ad = smem_desc_noswizzle(smem_u32(sQ) + ks * 256, 128, 16 * C_HEAD);
        const uint64_t bd = smem_desc_noswizzle(smem_u32(sK[s]) + ks * 256, 128, 16 * C_HEAD);
        umma_ss(tS, ad, bd, idS, ks > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    __syncwarp();
    mbar_wait(bar_mma, mph, status, DEV_TIMEOUT_MMA);
    __syncwarp();
    mph ^= 1;
    tc_fence_after();

    // ---- logits (log2 domain) and row max ----
    float x[TILE];
#pragma unroll
    for (int cch = 0; cch < 4; ++cch) {
      uint32_t sr[32];
      tmem_ld32(tmem_addr(tS, warp * 32, cch * 32), sr);
      tmem_ld_wait();
#pragma unroll
      for (int kk = 0; kk < 32; kk += 4) {
        const int k = cch * 32 + kk;
        const float4 t4 = __ldg(reinterpret_cast<const float4*>(tb + kt * TILE + k));
        const float4 m4 = *reinterpret_cast<const float4*>(sMB + kt * TILE + k);
        x[k + 0] = fmaf(__uint_as_float(sr[kk + 0]), c_l2, m4.x) + t4.x;
        x[k + 1] = fmaf(__uint_as_float(sr[kk + 1]), c_l2, m4.y) + t4.y;
        x[k + 2] = fmaf(__uint_as_float(sr[kk + 2]), c_l2, m4.z) + t4.z;
        x[k + 3] = fmaf(__uint_as_float(sr[kk + 3]), c_l2, m4.w) + t4.w;
      }
    }
    float rmax = x[0];
#pragma unroll
    for (int k = 1; k < TILE; ++k) rmax = fmaxf(rmax, x[k]);
    const float m_new = fmaxf(m, rmax);
    const float alpha = ex2(m - m_new);
    m = m_new;
    float sum = 0.f;
#pragma unroll
    for (int cch = 0; cch < 4; ++cch) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = ex2(x[cch * 32 + 2 * i] - m_new);
        const float p1 = ex2(x[cch * 32 + 2 * i + 1] - m_new);
        sum += p0 + p1;
        pk[i] = H16<T>::pack(p0, p1);
      }
      tmem_st16(tmem_addr(tS, warp * 32, cch * 16), pk);
    }
    tmem_st_wait();
    l = l * alpha + sum;
#pragma unroll
    for (int d = 0; d < C_HEAD; ++d) o[d] *= alpha;
    tc_fence_before();
    __syncthreads();

    // ---- O_part = P V ----
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < TILE / 16; ++j) {
        const uint64_t bd = smem_desc_noswizzle(smem_u32(sV[s]) + j * 1024, 512, 128);
        umma_ts(tO, tS + j * 8, bd, idO, j > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    __syncwarp();
    mbar_wait(bar_mma, mph, status, DEV_TIMEOUT_MMA);
    __syncwarp();
    mph ^= 1;
    tc_fence_after();
    {
      uint32_t orr[32];
      tmem_ld32(tmem_addr(tO, warp * 32, 0), orr);
      tmem_ld_wait();
#pragma unroll
      for (int d = 0; d < C_HEAD; ++d) o[d] += __uint_as_float(orr[d]);
    }
    tc_fence_before();
    // stage s is free (both MMAs that read it are complete): prefetch tile kt + 2
    if (tid == 0 && kt + 2 < NT) {
      mbar_arrive_expect_tx(bar_kv + s, 16384);
      bulk_g2s(sK[s], kimg + (size_t)(kt + 2) * 8192, 8192, bar_kv + s);
      bulk_g2s(sV[s], vimg + (size_t)(kt + 2) * 8192, 8192, bar_kv + s);
    }
  }

  // ---- epilogue: o / l * sigmoid(g) -> core operand image (tile (b, a, qt), channels h*32..) ----
  {
    const float inv_l = 1.0f / l;
    const T* g = reinterpret_cast<const T*>(args.ws + args.wl.off_g) + (((size_t)b * R + al) * N + qc) * C_IN + h * C_HEAD;
    unsigned char* cimg = args.ws + args.wl.off_core + (((size_t)b * R + al) * NT + qt) * 32768;
#pragma unroll
    for (int d = 0; d < C_HEAD; d += 8) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g + d);
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t ow[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 gg = H16<T>::unpack(gw[i]);
        const float y0 = o[d + 2 * i] * inv_l / (1.0f + __expf(-gg.x));
        const float y1 = o[d + 2 * i + 1] * inv_l / (1.0f + __expf(-gg.y));
        ow[i] = valid ? H16<T>::pack(y0, y1) : 0u;
      }
      *reinterpret_cast<uint4*>(cimg + img_off(tid, h * C_HEAD + d, HC)) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

template <typename T>
static cudaError_t core_tc_launch(const LayerArgs& a, cudaStream_t st) {
  // at least ~100 KB of shared memory per CTA: two CTAs per SM, matching the 2 x 256 TMEM columns
  const int smem = max(CORE_SMEM_FIXED + a.wl.Np * 4, 100 * 1024);
  cudaFuncSetAttribute(core_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int R = a.row_end - a.row_begin;
  dim3 grid(a.wl.NT, R, a.B * HEADS);
  core_tc_kernel<T><<<grid, 128, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_core_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  return dtype == DT_BF16 ? core_tc_launch<__nv_bfloat16>(a, st) : core_tc_launch<__half>(a, st);
}

// =================================================================================================
// Output projection (+ residual).  CTA = 128 pairs; y[128 x 128] = core[128 x 128] * W_o^T.
// =================================================================================================
constexpr int OP_SMEM = 65536 + 64;

template <typename T>
__global__ void __launch_bounds__(128) out_proj_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sA = smem;
  unsigned char* sW = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int ct = blockIdx.x, al = blockIdx.y, a = args.row_begin + al, b = blockIdx.z;
  const int N = args.N, R = args.row_end - args.row_begin, NT = args.wl.NT;
  int* status = args.status;
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
    mbar_arrive_expect_tx(bars + 0, 65536);
    bulk_g2s(sA, args.ws + args.wl.off_core + (((size_t)b * R + al) * NT + ct) * 32768, 32768, bars + 0);
    bulk_g2s(sW, args.packed + PackedLayout::img_o, 32768, bars + 0);
    mbar_wait(bars + 0, 0, status, DEV_TIMEOUT_TMA);
    tc_fence_after();
    constexpr uint32_t idesc = make_idesc_f16(128, 128, H16<T>::is_bf16, 0, 0);
#pragma unroll
    for (int ks = 0; ks < HC / 16; ++ks) {
      const uint64_t ad = smem_desc_noswizzle(smem_u32(sA) + ks * 256, 128, 16 * HC);
      const uint64_t bd = smem_desc_noswizzle(smem_u32(sW) + ks * 256, 128, 16 * HC);
      umma_ss(tbase, ad, bd, idesc, ks > 0 ? 1u : 0u);
    }
    umma_commit(bars + 1);
  }
  __syncwarp();
  mbar_wait(bars + 1, 0, status, DEV_TIMEOUT_MMA);
  __syncwarp();
  tc_fence_after();
  const int c = ct * TILE + tid;
  const bool valid = c < N;
  const long long ooff = b * args.ov.s_batch + (long long)(a - args.ov.row0) * args.ov.s_row + (long long)c * args.ov.s_col;
  const long long zoff = b * args.zv.s_batch + (long long)(a - args.zv.row0) * args.zv.s_row + (long long)c * args.zv.s_col;
#pragma unroll 1
  for (int cch = 0; cch < 4; ++cch) {
    uint32_t acc[32];
    tmem_ld32(tmem_addr(tbase, warp * 32, cch * 32), acc);
    tmem_ld_wait();
    if (valid) {
#pragma unroll
      for (int d = 0; d < 32; d += 4) {
        float4 y = make_float4(__uint_as_float(acc[d]), __uint_as_float(acc[d + 1]), __uint_as_float(acc[d + 2]),
                               __uint_as_float(acc[d + 3]));
        if (args.add_residual) {
          const float4 zz = *reinterpret_cast<const float4*>(args.z + zoff + cch * 32 + d);
          y.x += zz.x; y.y += zz.y; y.z += zz.z; y.w += zz.w;
        }
        *reinterpret_cast<float4*>(args.out + ooff + cch * 32 + d) = y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 128);
}

template <typename T>
static cudaError_t out_proj_tc_launch(const LayerArgs& a, cudaStream_t st) {
  cudaFuncSetAttribute(out_proj_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, OP_SMEM);
  const int R = a.row_end - a.row_begin;
  dim3 grid(a.wl.NT, R, a.B);
  out_proj_tc_kernel<T><<<grid, 128, OP_SMEM, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_out_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  return dtype == DT_BF16 ? out_proj_tc_launch<__nv_bfloat16>(a, st) : out_proj_tc_launch<__half>(a, st);
}

}  // namespace triattn
