// 16-bit (fp16 / bf16) path of the triangle-attention layer on the sm_100a tensor cores (tcgen05,
// accumulators in TMEM), fp32 accumulation / softmax statistics / residual.
//
// Data flow of one layer (attention orientation x[a][c]; ending node: x[a][c] = z[c][a], read in
// place through strides):
//   ln_proj_tc : z rows -> LN (fp32 stats) -> xn 16-bit operand image in smem -> UMMA with the
//                W_qkvg image (512 x 128) -> q (x C^-1/2 log2 e), k, v (fp16) operand images (8 KB per
//                128-position tile and head), g (row-major 16-bit); tri bias (fp32 SIMT dot from fp32
//                xn, x log2 e, stored fp16 in 128 x 128 blocks).
//   core_tc    : per (b, row a, head h, 128-query tile): S = Q K^T + tri bias x I (UMMA, SS) in TMEM ->
//                log2-domain logits (+ mask bias on mixed tiles), online softmax
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
// LN + q|k|v|g projection (+ tri bias).  Persistent: one CTA per SM (512 threads) loads the 128 KB
// weight image once and walks the 128-pair tiles (a, c0..c0+127) tile = blockIdx.x, + gridDim.x, ...
// Warp-specialised, so that the LayerNorm of one tile runs while the previous tile is written out:
//   LN group (warps 0..7): LayerNorm of tile i -> operand image i & 1 in shared memory (128-byte
//     swizzle) + tri-bias row sums; warp w holds pairs 16w..16w+15 in two passes of 8, four lanes per
//     pair (lane & 3 = qq: channels 16 j + 4 qq .. + 3, j = 0..7: a pair's four lanes load 64 contiguous
//     bytes at a time), so a statistic is a thread-local sum plus two shuffles and the four head sums of
//     the tri bias end one per lane after four shuffles; the LayerNorm affine and tri-bias weights are read
//     from shared memory.  The z rows of tile i + 1 are loaded into registers right after the LayerNorm of
//     tile i.
//     Warps 2 and 3 write the tile's tri-bias block once the group's row sums are complete.
//   drain group (warps 8..15): warp (part, quadrant) reads TMEM lanes 32 quadrant.. of half `part` and
//     writes q (x C^-1/2 log2 e) and k as K-major images, or v (MN-major image) and g (row-major, + gate
//     bias).  Warp 8 lane 0 issues the MMA D[128 x 512] = xn W^T of tile i in two N = 256 halves (q|k into
//     TMEM columns 0..255, v|g into 256..511) once image i is complete, each half as soon as that half of
//     tile i - 1 has been drained; one commit per half.
// TMEM: 512 columns = the full 128 x 512 fp32 accumulator of one tile.
// =================================================================================================
#ifndef TRIATTN_LP_LN_WARPS
#define TRIATTN_LP_LN_WARPS 8
#endif
constexpr int LP_LN_WARPS = TRIATTN_LP_LN_WARPS;                 // LayerNorm group: 8 or 16 pairs per warp
constexpr int LP_DRAIN_WARPS = LP_LN_WARPS == 8 ? 8 : 4;        // drain group: 4 warps per TMEM half, or 4 for both
constexpr int LP_PARTS = LP_DRAIN_WARPS / 4;                    // TMEM halves per drain warp: 2 -> 1 each, 1 -> both
constexpr int LP_THREADS = 32 * (LP_LN_WARPS + LP_DRAIN_WARPS);
constexpr int LP_W_BYTES = NPROJ * C_IN * 2;  // 131072
constexpr int LP_A_BYTES = TILE * C_IN * 2;   // 32768
constexpr int LP_SW = LP_W_BYTES + 2 * LP_A_BYTES + 2 * HEADS * TILE * 4 + C_IN * 4;  // ln_w, ln_b, w_b [4] (fp32)
constexpr int LP_SMEM = LP_SW + (2 + HEADS) * C_IN * 4 + 128;
#ifndef TRIATTN_LP_PREFETCH
#define TRIATTN_LP_PREFETCH 2
#endif
constexpr int LP_PREFETCH = TRIATTN_LP_PREFETCH;  // tiles whose rows are in L2 ahead of the register loads

template <typename T, bool XN, bool TB>
__global__ void __launch_bounds__(LP_THREADS, 1) ln_proj_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sW = smem;
  unsigned char* sA = smem + LP_W_BYTES;
  float* sBias = reinterpret_cast<float*>(smem + LP_W_BYTES + 2 * LP_A_BYTES);  // [2][4][128]
  float* sGb = reinterpret_cast<float*>(smem + LP_W_BYTES + 2 * LP_A_BYTES + 2 * HEADS * TILE * 4);  // g bias [128]
  float* sLw = reinterpret_cast<float*>(smem + LP_SW);  // [2 + HEADS][128]: ln_w, ln_b, w_b rows
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LP_SW + (2 + HEADS) * C_IN * 4);
  uint64_t* bar_w = bars;         // weight image landed
  uint64_t* bar_mma = bars + 1;   // [2] MMA half (q|k, v|g) of the current tile complete
  uint64_t* bar_tmem = bars + 3;  // [2] that half drained (4 warps each)
  uint64_t* bar_img = bars + 5;   // [2] every MMA reading operand image s complete
  uint64_t* bar_ready = bars + 7;  // [2] the LN group's operand image s is complete (one completion per use)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 9);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int N = args.N, R = args.row_end - args.row_begin, NT = args.wl.NT;
  const int ntiles = NT * R * args.B;
  const float* P = reinterpret_cast<const float*>(args.packed);
  int* status = args.status;

  // the swizzled operand image needs a 1024-byte aligned base (uniform over the CTA)
  if ((smem_u32(sA) & 1023u) != 0) {
    if (tid == 0) atomicCAS(status, 0, (int)DEV_BAD_ALIGN);
    return;
  }
  if (tid == 0) {
    mbar_init(bar_w, 1);
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar_mma + h, 1);
      mbar_init(bar_tmem + h, 4);
      mbar_init(bar_img + h, 1);
      mbar_init(bar_ready + h, 1);
    }
    fence_mbar_init();
  }
  if (tid < C_IN) sGb[tid] = P[PackedLayout::g_b / 4 + tid];
  for (int i = tid; i < (2 + HEADS) * C_IN; i += LP_THREADS)
    sLw[i] = i < C_IN ? P[PackedLayout::ln_w / 4 + i]
                      : (i < 2 * C_IN ? P[PackedLayout::ln_b / 4 + i - C_IN] : P[PackedLayout::w_b / 4 + i - 2 * C_IN]);
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  if (tid == 0 && (int)blockIdx.x < ntiles) {
    mbar_arrive_expect_tx(bar_w, LP_W_BYTES);
    bulk_g2s(sW, args.packed + PackedLayout::img_qkvg, LP_W_BYTES, bar_w);
  }
  // caller-given LayerNorm output (16-bit, this layer's type): the LN is skipped and its bits become
  // the operand image as they are (kernel-uniform)
  constexpr bool xn_mode = XN;
  // the producer of xn also gave this layer's tri bias (args.tb_in): the SIMT tri-bias dot is skipped
  constexpr bool tb_given = XN && TB;

    // the z (or xn) rows of a tile pulled into L2 ahead of their register loads: rows that are contiguous
    // in memory (a dense view whose columns are consecutive pairs) as one bulk prefetch, otherwise one
    // bulk prefetch per row (512 B of fp32 z, 256 B of 16-bit xn) spread over the drain group's threads (the bulk-copy unit takes them one at a time, off the
    // LayerNorm group's path)
    const View& pv = xn_mode ? args.xnv : args.zv;
    const bool rows_contiguous = !pv.cblk && pv.s_col == C_IN;
    constexpr int ROW_BYTES = xn_mode ? C_IN * 2 : C_IN * 4;
    auto prefetch_rows = [&](int tile, int e) {  // e: this thread's index in the issuing group
      if (tile >= ntiles) return;
      const int ct = tile % NT, al = (tile / NT) % R, b = tile / (NT * R);
      const unsigned char* base =
          (xn_mode ? static_cast<const unsigned char*>(args.xn) : reinterpret_cast<const unsigned char*>(args.z)) +
          (b * pv.s_batch + (long long)(args.row_begin + al - pv.row0) * pv.s_row) * (ROW_BYTES / C_IN);
      const int c0 = ct * TILE, rows = min(TILE, N - c0);
      if (rows_contiguous) {
        if (e == 0) prefetch_l2_bulk(base + (long long)c0 * ROW_BYTES, rows * ROW_BYTES);
      } else if (e < rows) {
        prefetch_l2_bulk(base + view_col(pv, c0 + e) * (ROW_BYTES / C_IN), ROW_BYTES);
      }
    };
  if (warp < LP_LN_WARPS) {
    // ================================ LN group ================================
    const int qq = lane & 3;
    constexpr int PASSES = 128 / (8 * LP_LN_WARPS);  // groups of 8 pairs per warp
    // rows (PASSES warp + pass) 8 + lane / 4 of a tile: xv[pass][j] = channels 16 j + 4 qq .. + 3 (zeros
    // past N; xn mode: 4 16-bit values in .x / .y)
    auto load_rows = [&](int tile, int ps, float4 (&xvp)[8]) {
      const int ct = tile % NT, al = (tile / NT) % R, b = tile / (NT * R);
      {
        const int c = ct * TILE + 8 * (PASSES * warp + ps) + (lane >> 2);
        if constexpr (xn_mode) {
          const uint16_t* xr = reinterpret_cast<const uint16_t*>(args.xn) + b * args.xnv.s_batch +
                               (long long)(args.row_begin + al - args.xnv.row0) * args.xnv.s_row;
          const uint2* src = reinterpret_cast<const uint2*>(xr + (c < N ? view_col(args.xnv, c) : 0)) + qq;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint2 u = c < N ? __ldcs(src + 4 * j) : make_uint2(0u, 0u);
            xvp[j] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), 0.f, 0.f);
          }
        } else {
          const float* zr =
              args.z + b * args.zv.s_batch + (long long)(args.row_begin + al - args.zv.row0) * args.zv.s_row;
          const float4* src = reinterpret_cast<const float4*>(zr + (c < N ? view_col(args.zv, c) : 0)) + qq;
#pragma unroll
          for (int j = 0; j < 8; ++j) xvp[j] = c < N ? __ldcs(src + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    };
    auto ln_rows = [&](int it, int ps, const float4 (&xv)[8]) {
      float* sB = sBias + (it & 1) * HEADS * TILE;
      unsigned char* sAi = sA + (it & 1) * LP_A_BYTES;
      const int rw = 8 * (PASSES * warp + ps) + (lane >> 2);
      const float4* w4 = reinterpret_cast<const float4*>(sLw) + qq;  // row q of sLw: w4[32 q + 4 j]
      // packed fp32 pairs (f32x2 instructions): a = channels (16 j + 4 qq, + 1), b = (+ 2, + 3)
      auto lo = [](const float4& v) { return make_float2(v.x, v.y); };
      auto hi = [](const float4& v) { return make_float2(v.z, v.w); };
      float2 nmean = make_float2(0.f, 0.f), rstd2 = make_float2(0.f, 0.f);
      if constexpr (!xn_mode) {
        float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) s2 = __fadd2_rn(s2, __fadd2_rn(lo(xv[j]), hi(xv[j])));
        float s = s2.x + s2.y;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        const float mean = s * (1.0f / C_IN);
        nmean = make_float2(-mean, -mean);
        float2 v2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 da = __fadd2_rn(lo(xv[j]), nmean), db = __fadd2_rn(hi(xv[j]), nmean);
          v2 = __ffma2_rn(da, da, v2);
          v2 = __ffma2_rn(db, db, v2);
        }
        float v = v2.x + v2.y;
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        const float rstd = rsqrtf(v * (1.0f / C_IN) + LN_EPS);
        rstd2 = make_float2(rstd, rstd);
      }
      // head sums as pairs (even, odd channel), added up at the end
      float2 p2[HEADS] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float2 na, nb;
        uint2 pk;
        if constexpr (xn_mode) {
          pk = make_uint2(__float_as_uint(xv[j].x), __float_as_uint(xv[j].y));
          na = H16<T>::unpack(pk.x);
          nb = H16<T>::unpack(pk.y);
        } else {
          const float4 lw = w4[4 * j], lb = w4[32 + 4 * j];
          na = __ffma2_rn(__fmul2_rn(__fadd2_rn(lo(xv[j]), nmean), rstd2), lo(lw), lo(lb));
          nb = __ffma2_rn(__fmul2_rn(__fadd2_rn(hi(xv[j]), nmean), rstd2), hi(lw), hi(lb));
          pk.x = H16<T>::pack(na.x, na.y);
          pk.y = H16<T>::pack(nb.x, nb.y);
        }
        // swizzled image: the 8 bytes of channels 16 j + 4 qq .. + 3 of row rw
        *reinterpret_cast<uint2*>(sAi + sw128_off(rw, 16 * j + 4 * qq, LP_A_BYTES / 2)) = pk;
        if constexpr (!tb_given) {
#pragma unroll
          for (int hh = 0; hh < HEADS; ++hh) {
            const float4 wb = w4[32 * (2 + hh) + 4 * j];
            p2[hh] = __ffma2_rn(na, lo(wb), p2[hh]);
            p2[hh] = __ffma2_rn(nb, hi(wb), p2[hh]);
          }
        }
      }
      float p[HEADS];
#pragma unroll
      for (int hh = 0; hh < HEADS; ++hh) p[hh] = p2[hh].x + p2[hh].y;
      if constexpr (!tb_given) {
        // the row's four head sums over its four lanes: exchange halves (xor 2: heads 0,1 | 2,3), then one
        // head each (xor 1); lane qq ends with head qq's total
        const bool up2 = qq & 2, up1 = qq & 1;
        float k0 = up2 ? p[2] : p[0], k1 = up2 ? p[3] : p[1];
        k0 += __shfl_xor_sync(0xffffffffu, up2 ? p[0] : p[2], 2);
        k1 += __shfl_xor_sync(0xffffffffu, up2 ? p[1] : p[3], 2);
        float k = up1 ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, up1 ? k0 : k1, 1);
        sB[qq * TILE + rw] = k;
      }
    };
    float4 xv[PASSES][8];
    int tile = blockIdx.x;
    if (tile < ntiles)
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps) load_rows(tile, ps, xv[ps]);
    for (int it = 0; tile < ntiles; tile += gridDim.x, ++it) {
      // operand image it & 1 is free once every MMA of tile it - 2 has completed (tri-bias slot it & 1 was
      // last read by warps 2, 3 before the group barrier of tile it - 1)
      if (it >= 2) mbar_wait(bar_img + (it & 1), ((it >> 1) - 1) & 1, status, DEV_TIMEOUT_MMA);
      // each pass's registers take the next tile's rows as soon as the pass is done (in flight for a tile)
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps) {
        ln_rows(it, ps, xv[ps]);
        if (tile + (int)gridDim.x < ntiles) load_rows(tile + gridDim.x, ps, xv[ps]);
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;" ::"n"(32 * LP_LN_WARPS) : "memory");  // the group's image and tri-bias sums are complete
      // ---- tri-bias rows of attention row a (warps 2, 3): fp16, log2 domain, 128 x 128 block layout
      //      [k/8][q][8]; one 16-byte chunk = 8 consecutive keys of one head (padded keys 0); a
      //      producer-given tri bias: fp16 [B][HEADS][N][N], element (b, hh, a, c) ----
      if (warp == 2 || warp == 3) {
        const int ct = tile % NT, al = (tile / NT) % R, b = tile / (NT * R);
        const int a = args.row_begin + al, c0 = ct * TILE;
        const float* sB = sBias + (it & 1) * HEADS * TILE;
        const int t64 = tid - 64, hh = t64 / (TILE / 8), kg = t64 % (TILE / 8);
        const __half* tbr =
            tb_given ? static_cast<const __half*>(args.tb_in) + (((size_t)b * HEADS + hh) * N + a) * N : nullptr;
        auto bias_at = [&](int r0) -> float {
          if (c0 + r0 >= N) return 0.0f;
          return (tb_given ? __half2float(tbr[c0 + r0]) : sB[hh * TILE + r0]) * LOG2E;
        };
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r0 = kg * 8 + 2 * i;
          w[i] = H16<__half>::pack(bias_at(r0), bias_at(r0 + 1));
        }
        *reinterpret_cast<uint4*>(args.ws + args.wl.off_bias + bias16_off(a, c0 + kg * 8, b, hh, args.B, NT)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (tid == 0) mbar_arrive(bar_ready + (it & 1));
    }
  } else {
    // ================================ drain group ================================
    const int quad = warp & 3;  // TMEM lanes 32 quad..
    const int e = tid - 32 * LP_LN_WARPS;
#pragma unroll 1
    for (int d = 1; d <= LP_PREFETCH; ++d) prefetch_rows(blockIdx.x + d * gridDim.x, e);
    // TMEM halves this warp drains: [p0, p1)
    const int p0 = LP_PARTS == 2 ? (warp - LP_LN_WARPS) >> 2 : 0, p1 = LP_PARTS == 2 ? p0 + 1 : 2;
    int tile = blockIdx.x;
    for (int it = 0; tile < ntiles; tile += gridDim.x, ++it) {
      prefetch_rows(tile + (LP_PREFETCH + 1) * gridDim.x, e);
      if (warp == LP_LN_WARPS) {
        if (lane == 0) {
          mbar_wait(bar_ready + (it & 1), (it >> 1) & 1, status, DEV_TIMEOUT_SYNC);
          if (it == 0) mbar_wait(bar_w, 0, status, DEV_TIMEOUT_TMA);
          unsigned char* sAi = sA + (it & 1) * LP_A_BYTES;
          constexpr uint32_t idesc = make_idesc_f16(128, 256, H16<T>::is_bf16, 0, 0);
#pragma unroll
          for (int nh = 0; nh < 2; ++nh) {
            if (it > 0) mbar_wait(bar_tmem + nh, (it - 1) & 1, status, DEV_TIMEOUT_SYNC);  // half nh of tile it - 1 drained
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < C_IN / 16; ++ks) {
              const uint64_t ad = smem_desc_sw128(smem_u32(sAi) + (ks / 4) * (LP_A_BYTES / 2) + (ks % 4) * 32);
              const uint64_t bd = smem_desc_noswizzle(smem_u32(sW) + nh * 65536 + ks * 256, 128, 16 * C_IN);
              umma_ss(tbase + nh * 256, ad, bd, idesc, ks > 0 ? 1u : 0u);
            }
            umma_commit(bar_mma + nh);
          }
          umma_commit(bar_img + (it & 1));
        }
        __syncwarp();
      }
      const int ct = tile % NT, al = (tile / NT) % R, b = tile / (NT * R);
      const int c0 = ct * TILE;
      const int r = quad * 32 + lane, c = c0 + r;
      const bool valid = c < N;
#pragma unroll 1
      for (int part = p0; part < p1; ++part) {  // TMEM half: q|k, v|g
      mbar_wait(bar_mma + part, it & 1, status, DEV_TIMEOUT_MMA);
      __syncwarp();
      tc_fence_after();
#pragma unroll 1
      for (int sub = 0; sub < 2; ++sub) {
        const int tt = 2 * part + sub;  // 0 q, 1 k, 2 v, 3 g
#pragma unroll 1
        for (int hh = 0; hh < HEADS; ++hh) {
          uint32_t acc[32];
          tmem_ld32(tmem_addr(tbase, quad * 32, tt * 128 + hh * 32), acc);
          tmem_ld_wait();
          tmem_regs_ready(acc);
          if (tt <= 1) {
            // q (pre-scaled by C^-1/2 log2 e: the core's S is then in log2 units) and k: K-major images
            const float sc = tt == 0 ? QSCALE_L2 : 1.0f;
            const float2 sc2 = make_float2(sc, sc);
            unsigned char* img = args.ws + (tt == 0 ? args.wl.off_q : args.wl.off_k) +
                                 ((((size_t)b * R + al) * HEADS + hh) * NT + ct) * 8192;
            auto qk2 = [&](int i) {
              const float2 v = __fmul2_rn(make_float2(__uint_as_float(acc[i]), __uint_as_float(acc[i + 1])), sc2);
              return H16<T>::pack(v.x, v.y);
            };
#pragma unroll
            for (int d = 0; d < C_HEAD; d += 8) {
              uint4 pk = make_uint4(0u, 0u, 0u, 0u);
              if (valid) pk = make_uint4(qk2(d), qk2(d + 2), qk2(d + 4), qk2(d + 6));
              *reinterpret_cast<uint4*>(img + img_off(r, d, C_HEAD)) = pk;
            }
          } else if (tt == 2) {
            // v: fp16 in every 16-bit mode (the P.V product runs in fp16), saturated to the fp16 range,
            // MN-major image read by the P.V MMA
            unsigned char* img = args.ws + args.wl.off_v + ((((size_t)b * R + al) * HEADS + hh) * NT + ct) * 8192;
            // fp16 pair (low half = acc[i]) rounded to nearest and saturated to the finite fp16 range
            auto sat2 = [&](int i) {
              uint32_t r;
              asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "r"(acc[i + 1]), "r"(acc[i]));
              return r;
            };
#pragma unroll
            for (int d = 0; d < C_HEAD; d += 8) {
              uint4 pk = make_uint4(0u, 0u, 0u, 0u);
              if (valid) pk = make_uint4(sat2(d), sat2(d + 2), sat2(d + 4), sat2(d + 6));
              *reinterpret_cast<uint4*>(img + vimg_off(r, d)) = pk;
            }
          } else if (valid) {
            const float2* gb = reinterpret_cast<const float2*>(sGb + hh * C_HEAD);
            T* g = reinterpret_cast<T*>(args.ws + args.wl.off_g) + (((size_t)b * R + al) * N + c) * C_IN + hh * C_HEAD;
            auto g2 = [&](int i) {
              const float2 v = __fadd2_rn(make_float2(__uint_as_float(acc[i]), __uint_as_float(acc[i + 1])), gb[i / 2]);
              return H16<T>::pack(v.x, v.y);
            };
#pragma unroll
            for (int d = 0; d < C_HEAD; d += 8)
              *reinterpret_cast<uint4*>(g + d) = make_uint4(g2(d), g2(d + 2), g2(d + 4), g2(d + 6));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tmem + part);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

template <typename T, bool XN, bool TB = false>
static cudaError_t ln_proj_tc_launch(const LayerArgs& a, cudaStream_t st) {
  cudaFuncSetAttribute(ln_proj_tc_kernel<T, XN, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, LP_SMEM);
  const int ntiles = a.wl.NT * (a.row_end - a.row_begin) * a.B;
  const int grid = ntiles < a.num_sms ? ntiles : a.num_sms;
  ln_proj_tc_kernel<T, XN, TB><<<grid, LP_THREADS, LP_SMEM, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ln_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  if (a.xn && a.tb_in)
    return dtype == DT_BF16 ? ln_proj_tc_launch<__nv_bfloat16, true, true>(a, st)
                            : ln_proj_tc_launch<__half, true, true>(a, st);
  if (a.xn) return dtype == DT_BF16 ? ln_proj_tc_launch<__nv_bfloat16, true>(a, st) : ln_proj_tc_launch<__half, true>(a, st);
  return dtype == DT_BF16 ? ln_proj_tc_launch<__nv_bfloat16, false>(a, st) : ln_proj_tc_launch<__half, false>(a, st);
}

// =================================================================================================
// Mask bias + key-tile classes (16-bit path).  One CTA per (attention row, batch), 128 threads.
//   mb[b][row][k] = log2(e) * inf * (mask - 1)  (k < N),  -1e30 for padded keys
//   ts[b][row][kt] (row stride NTs) = 0 every key of the tile valid, 1 every key masked and the row has a valid key
//   elsewhere (the tile contributes exactly 0 and is skipped), 2 otherwise (mask bias applied; a
//   row with no valid key at all keeps every tile, which makes it attend uniformly, as in fp32).
// =================================================================================================
__global__ void __launch_bounds__(128) mask_prep_tc_kernel(LayerArgs args) {
  __shared__ uint8_t cls[TILE];  // NT <= 128 (N <= 16384)
  __shared__ int any_valid;
  const int tid = threadIdx.x;
  const int al = blockIdx.x, a = args.row_begin + al, b = blockIdx.y;
  const int N = args.N, R = args.row_end - args.row_begin, Np = args.wl.Np, NT = args.wl.NT;
  float* mb = reinterpret_cast<float*>(args.ws + args.wl.off_mb) + ((size_t)b * R + al) * Np;
  if (tid == 0) any_valid = 0;
  __syncthreads();
  const View mv = args.mv;
  for (int kt = 0; kt < NT; ++kt) {
    const int k = kt * TILE + tid;
    float v = -1e30f;
    if (k < N) {
      const float m =
          args.mask ? args.mask[b * mv.s_batch + (long long)(a - mv.row0) * mv.s_row + view_col(mv, k)] : 1.0f;
      v = args.inf * (m - 1.0f) * LOG2E;
    }
    mb[k] = v;
    const int n_valid = __syncthreads_count(k < N && v == 0.0f);
    const int n_bad = __syncthreads_count(!(k < N && v == 0.0f));
    if (tid == 0) {
      cls[kt] = n_valid == 0 ? 1 : (n_bad == 0 ? 0 : 2);
      if (n_valid) any_valid = 1;
    }
  }
  __syncthreads();
  uint8_t* ts = args.ws + args.wl.off_ts + ((size_t)b * R + al) * args.wl.NTs;
  for (int kt = tid; kt < NT; kt += blockDim.x) ts[kt] = any_valid ? cls[kt] : 2;
}

cudaError_t launch_mask_prep_tc(const LayerArgs& a, cudaStream_t st) {
  dim3 grid(a.row_end - a.row_begin, a.B);
  mask_prep_tc_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}

// =================================================================================================
// Flash core, persistent.  A work item = (batch b, head h, 128-query tile qt, pair of attention
// rows); items are numbered with qt fastest (CTAs running at the same time read the same rows' K/V
// tiles, which stay in L2) and CTA c takes items c, c + gridDim.x, ...  Two CTAs share each SM
// (2 x 92 KB shared memory, 2 x 256 TMEM columns, 2 x 256 threads at 128 registers): each has its
// own tri-bias stage, so the two drift out of phase and one's MMA waits overlap the other's softmax
// (one CTA of four rows keeps its rows in lockstep through the shared stage: 8 % slower).  The
// tri-bias tile of (h, qt, kt) is loaded once per key tile and shared by the CTA's rows.
//   8 warps = two softmax warpgroups; warpgroup j owns row j of the item (TMEM lanes = queries).
//   Each row's leader thread issues that row's work itself: the bulk copies of its Q, K and V tiles
//   (one slot each, refilled as soon as the MMA that read the slot has completed; after the row's
//   last tile of an item they are refilled with the first active tile of the row's next item) and
//   its MMAs (S = Q K^T + tri bias, then O = P V).  The tri bias is added on the tensor pipe: the fp16
//   bias block of the stage, already a K-major operand image, against a 64 x 64 identity, one MMA per
//   64-key half and K step of 16, accumulating exactly onto S.  The tri-bias stage is refilled by
//   whichever warp is the last of the CTA's 8 to finish with it (an arrival counter in shared memory).
// TMEM (256 columns): row j owns columns [128 j, 128 j + 128): S (fp32, log2 units, tri bias included;
// mixed tiles: + mask bias, written back) -> P (fp16 pairs in columns 0..63) and the P.V partial
// (columns 64..111: 32 channels + the row sum from V's ones column).  O is accumulated in registers
// with a lazy rescale.
// =================================================================================================
constexpr int CG_RG = 2;            // rows per CTA; two CTAs share an SM
constexpr int CG_SOFTMAX_WARPS = 4 * CG_RG;
constexpr int CG_THREADS = CG_SOFTMAX_WARPS * 32;
constexpr int CG_NB = 1;                           // tri-bias stages
constexpr int CG_SQ = 0;                           // RG Q tiles, 8 KB each
constexpr int CG_SB = CG_SQ + CG_RG * 8192;        // NB tri-bias stages, 32 KB each (fp16)
constexpr int CG_SMB = CG_SB + CG_NB * 32768;      // NB stages x RG mask-bias slices of 512 B
constexpr int CG_SK = CG_SMB + CG_NB * CG_RG * 512;  // one K slot per row, 8 KB
constexpr int CG_SV = CG_SK + CG_RG * 8192;        // one V slot per row, 12 KB (8 KB V + 4 KB ones/zeros)
constexpr int CG_SI = CG_SV + CG_RG * 12288;        // 64 x 64 fp16 identity (K-major image, 8 KB): the tri-bias MMA's B
constexpr int CG_BAR = CG_SI + 8192;
constexpr int CG_CLS = CG_BAR + 512;               // 2 (item parity) x RG x 128 key-tile classes
constexpr int CG_CNT = CG_CLS + 2 * CG_RG * TILE;  // NB tri-bias stage arrival counters
constexpr int CG_RS = CG_CNT + 16;                 // RG row states (32 B each)
constexpr int CG_II = CG_RS + CG_RG * 32;          // 3 item-info slots (32 B each)
constexpr int CG_SMEM = CG_II + 3 * 32;
static_assert(2 * (CG_SMEM + 1024) <= 233472, "two core CTAs per SM");

// barrier slots
constexpr int B_BF = 0, B_QF = CG_NB, B_KF = B_QF + CG_RG, B_VF = B_KF + CG_RG, B_SF = B_VF + CG_RG,
              B_OF = B_SF + CG_RG, B_COUNT = B_OF + CG_RG;
static_assert(B_COUNT * 8 + 16 <= 512, "barrier area");

// Per-row state kept by the row's leader: K/V/Q tile indices (global tile = base + kt) of the
// current and the next item, the next item's query tile and its first active key tile.
struct CoreRowState {
  unsigned long long cur, nxt;
  int nxt_qt, nxt_first;
};
// Per-item bias addressing: byte offsets of the tri-bias block (h, qt) and of the mask-bias row of
// the group's first row; rows of the group inside the range (0 = no such item).
struct CoreItemInfo {
  unsigned long long bias_off, mb_off;
  int nrow, pad;
};

// Work item -> (b, h, qt, first row of the group).
struct CoreItem {
  int b, h, qt, g0;
};
__device__ __forceinline__ CoreItem core_item(int item, int NT, int G) {
  CoreItem it;
  it.qt = item % NT;
  const int rest = item / NT;
  it.g0 = (rest % G) * CG_RG;
  const int bh = rest / G;
  it.b = bh / HEADS;
  it.h = bh % HEADS;
  return it;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^(x0 - m), 2^(x1 - m) as an fp16 pair (low half x0): one packed fp32 subtract, two fp32 MUFU
// exponentials, one conversion to an fp16 pair.  The exponent stays fp32 up to the MUFU (a packed
// 16-bit exponential would round x - m to fp16 first: 2^-7 absolute at |x - m| = 16); the MUFU pipe
// time is the same (ex2.f16x2 takes two slots) and the core measured 0.7 % faster this way.
__device__ __forceinline__ uint32_t exp2_pair_f16(float x0, float x1, uint64_t neg_m2) {
  uint32_t r;
  asm("{\n\t.reg .b64 d;\n\t.reg .f32 a, b;\n\t"
      "mov.b64 d, {%1, %2};\n\tadd.rn.f32x2 d, d, %3;\n\tmov.b64 {a, b}, d;\n\t"
      "ex2.approx.ftz.f32 a, a;\n\tex2.approx.ftz.f32 b, b;\n\tcvt.rn.f16x2.f32 %0, b, a;\n\t}"
      : "=r"(r)
      : "f"(x0), "f"(x1), "l"(neg_m2));
  return r;
}

// 2^(x0 - m), 2^(x1 - m) as an fp16 pair computed without the MUFU (FMA and ALU pipes only), so a
// share of the exponentials runs beside the MUFU ones.  Cody-Waite style split: y = max(x - m, -32),
// n = round(y) with the 1.5 * 2^23 shifter, f = y - n in [-0.5, 0.5], 2^f from a degree-3
// polynomial fitted to 2^f on [-0.5, 0.5] by iteratively reweighted least squares on the relative
// error (max relative error 7.5e-5, below the fp16 rounding of P), then 2^y = 2^f * 2^n by adding
// n to the exponent field.
__device__ __forceinline__ uint32_t exp2_pair_poly_f16(float x0, float x1, uint64_t neg_m2) {
  constexpr float kC0 = 0x1.fff696p-1f, kC1 = 0x1.62f31ap-1f, kC2 = 0x1.f0dd6ep-3f, kC3 = 0x1.c3f60cp-5f;
  const uint64_t sh2 = 0x4B4000004B400000ull;  // (1.5 * 2^23, 1.5 * 2^23)
  const uint64_t c3 = ((uint64_t)__float_as_uint(kC3) << 32) | __float_as_uint(kC3);
  const uint64_t c2 = ((uint64_t)__float_as_uint(kC2) << 32) | __float_as_uint(kC2);
  const uint64_t c1 = ((uint64_t)__float_as_uint(kC1) << 32) | __float_as_uint(kC1);
  const uint64_t c0 = ((uint64_t)__float_as_uint(kC0) << 32) | __float_as_uint(kC0);
  float y0, y1;
  asm("{\n\t.reg .b64 d;\n\tmov.b64 d, {%2, %3};\n\tadd.rn.f32x2 d, d, %4;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(y0), "=f"(y1)
      : "f"(x0), "f"(x1), "l"(neg_m2));
  y0 = fmaxf(y0, -32.0f);
  y1 = fmaxf(y1, -32.0f);
  uint32_t t0, t1, p0, p1;
  asm("{\n\t.reg .b64 y, t, n, f, p;\n\t"
      "mov.b64 y, {%4, %5};\n\t"
      "add.rn.f32x2 t, y, %6;\n\t"
      "sub.rn.f32x2 n, t, %6;\n\t"
      "sub.rn.f32x2 f, y, n;\n\t"
      "fma.rn.f32x2 p, %7, f, %8;\n\t"
      "fma.rn.f32x2 p, p, f, %9;\n\t"
      "fma.rn.f32x2 p, p, f, %10;\n\t"
      "mov.b64 {%0, %1}, t;\n\tmov.b64 {%2, %3}, p;\n\t}"
      : "=r"(t0), "=r"(t1), "=r"(p0), "=r"(p1)
      : "f"(y0), "f"(y1), "l"(sh2), "l"(c3), "l"(c2), "l"(c1), "l"(c0));
  const float e0 = __uint_as_float(p0 + (t0 << 23));
  const float e1 = __uint_as_float(p1 + (t1 << 23));
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(e1), "f"(e0));
  return r;
}

// Named barrier of one softmax warpgroup (ids 1..RG; 0 is __syncthreads).
__device__ __forceinline__ void wg_sync(int j) { asm volatile("bar.sync %0, 128;" ::"r"(j + 1) : "memory"); }

template <typename T>
__global__ void __launch_bounds__(CG_THREADS, 2) core_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + CG_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + CG_BAR + B_COUNT * 8);
  uint8_t* scls = smem + CG_CLS;  // [item parity][row][kt]
  int* bias_cnt = reinterpret_cast<int*>(smem + CG_CNT);
  CoreItemInfo* iinfo = reinterpret_cast<CoreItemInfo*>(smem + CG_II);  // [item ordinal % 3]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = args.N, R = args.row_end - args.row_begin, NT = args.wl.NT, Np = args.wl.Np, NTs = args.wl.NTs;
  const int G = (R + CG_RG - 1) / CG_RG;
  const int n_items = NT * G * args.B * HEADS;
  int* status = args.status;
  const unsigned char* ts_all = args.ws + args.wl.off_ts;
  // key-tile classes kt = 4 w4 .. 4 w4 + 3 of row g0 + jj of an item, one byte each: 0 all valid,
  // 1 skip, 2 mixed; 3 = no such tile, row or item
  auto class_word = [&](int item, int jj, int w4) -> uint32_t {
    if (item >= n_items || 4 * w4 >= NTs) return 0x03030303u;
    const CoreItem ci = core_item(item, NT, G);
    if (ci.g0 + jj >= R) return 0x03030303u;
    uint32_t w = *reinterpret_cast<const uint32_t*>(ts_all + ((size_t)ci.b * R + ci.g0 + jj) * NTs + 4 * w4);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (4 * w4 + i >= NT) w = (w & ~(0xFFu << (8 * i))) | (3u << (8 * i));
    return w;
  };
  auto item_info = [&](int item) {
    CoreItemInfo f{};
    if (item < n_items) {
      const CoreItem ci = core_item(item, NT, G);
      f.bias_off = args.wl.off_bias + (((unsigned long long)ci.qt * args.B + ci.b) * HEADS + ci.h) * NT * 32768ull;
      f.mb_off = args.wl.off_mb + ((unsigned long long)ci.b * R + ci.g0) * Np * 4ull;
      f.nrow = min(CG_RG, R - ci.g0);
    }
    return f;
  };

  // ---- set-up (once per CTA): barriers, V-slot tails, classes of the first item, TMEM ----
  if (tid == 0) {
    for (int i = 0; i < CG_NB; ++i) mbar_init(bar + B_BF + i, 1);
    for (int j = 0; j < CG_RG; ++j) {
      mbar_init(bar + B_QF + j, 1);
      mbar_init(bar + B_KF + j, 1);
      mbar_init(bar + B_VF + j, 1);
      mbar_init(bar + B_SF + j, 1);
      mbar_init(bar + B_OF + j, 1);
    }
    for (int i = 0; i < CG_NB; ++i) bias_cnt[i] = 0;
    iinfo[0] = item_info(blockIdx.x);
    iinfo[1] = item_info(blockIdx.x + gridDim.x);
    fence_mbar_init();
  }
  // V slot tail: channel group 4 = (1, 0, ..., 0) per key (the ones column that yields the row
  // sum), channel group 5 = zeros.  2 x 2 KB per slot, never overwritten by the V copies.
  for (int i = tid; i < CG_RG * 1024; i += CG_THREADS) {
    const int stg = i / 1024, w = i % 1024;
    uint32_t* tail = reinterpret_cast<uint32_t*>(smem + CG_SV + stg * 12288 + 8192);
    tail[w] = (w < 512 && (w & 3) == 0) ? 0x00003C00u : 0u;  // fp16 1.0 in the low half of each key's first word
  }
  // identity image: element (n, j) of the K-major no-swizzle layout (LBO 128 B, SBO 1024 B) is fp16 1.0 iff n == j
  for (int e = tid; e < 4096; e += CG_THREADS) {
    const int byte = 2 * e, n = (byte >> 10) * 8 + ((byte & 127) >> 4), jj = ((byte & 1023) >> 7) * 8 + ((byte & 15) >> 1);
    reinterpret_cast<uint16_t*>(smem + CG_SI)[e] = n == jj ? 0x3C00u : 0u;
  }
  if (tid < CG_RG * 32)
    reinterpret_cast<uint32_t*>(scls)[tid] = class_word(blockIdx.x, tid / 32, tid % 32);
  fence_proxy_async_smem();
  if (warp == 0) tmem_alloc(tslot, CG_RG * 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // tri-bias tile kt of item ordinal i (+ the mask-bias slices of the item's rows) -> stage s % NB,
  // s = i * NT + kt; item infos of ordinals ii and ii + 1 are in their slots while item ii runs
  auto load_bias = [&](int i, int kt, int ii_now) {
    const int s = i * NT + kt;
    const CoreItemInfo f = (i <= ii_now + 1) ? iinfo[i % 3] : item_info(blockIdx.x + i * gridDim.x);
    if (f.nrow == 0) return;
    const int bs = s % CG_NB;
    mbar_arrive_expect_tx(bar + B_BF + bs, 32768 + f.nrow * 512);
    bulk_g2s(smem + CG_SB + bs * 32768, args.ws + f.bias_off + (size_t)kt * 32768, 32768, bar + B_BF + bs);
    for (int jj = 0; jj < f.nrow; ++jj)
      bulk_g2s(smem + CG_SMB + (bs * CG_RG + jj) * 512, args.ws + f.mb_off + ((size_t)jj * Np + kt * TILE) * 4, 512,
               bar + B_BF + bs);
  };
  if (tid == 0)
    for (int s = 0; s < CG_NB; ++s) load_bias(s / NT, s % NT, 0);

  // ================================ softmax warpgroups ================================
  const int j = warp >> 2, quad = warp & 3;  // row of the item, TMEM lane quadrant
  const int t = quad * 32 + lane;            // query within the tile = TMEM lane
  const bool leader = (quad == 0 && lane == 0);
  const uint32_t buf = tbase + ((uint32_t)(quad * 32) << 16) + j * 128;
  const uint32_t buf0 = tbase + j * 128;  // lane 0 of the row's columns (MMA operands)
  constexpr uint32_t idS = make_idesc_f16(128, 128, H16<T>::is_bf16, 0, 0);
  constexpr uint32_t idPV = make_idesc_f16(128, 48, 0, 0, 1);  // fp16 P (TMEM) x fp16 V (MN-major), N = 32 + 16
  constexpr uint32_t idB = make_idesc_f16(128, 64, 0, 0, 0);   // fp16 tri bias x fp16 identity, N = 64 keys
  CoreRowState* rs = reinterpret_cast<CoreRowState*>(smem + CG_RS) + j;
  // first active key tile >= kt of row j in the item whose classes are in slot cs
  auto next_active = [&](int cs, int kt) {
    const uint8_t* c = scls + (cs * CG_RG + j) * TILE;
    while (kt < NT && c[kt] != 0 && c[kt] != 2) ++kt;
    return kt;
  };
  // global tile index base of (row j of item): K/V/Q tiles at (base + kt) * 8192
  auto tile_base = [&](int item) -> unsigned long long {
    const CoreItem ci = core_item(item, NT, G);
    return ((((unsigned long long)ci.b * R) + ci.g0 + j) * HEADS + ci.h) * NT;
  };
  auto load_q = [&](unsigned long long tile) {
    mbar_arrive_expect_tx(bar + B_QF + j, 8192);
    bulk_g2s(smem + CG_SQ + j * 8192, args.ws + args.wl.off_q + tile * 8192, 8192, bar + B_QF + j);
  };
  auto load_k = [&](unsigned long long tile) {
    mbar_arrive_expect_tx(bar + B_KF + j, 8192);
    bulk_g2s(smem + CG_SK + j * 8192, args.ws + args.wl.off_k + tile * 8192, 8192, bar + B_KF + j);
  };
  auto load_v = [&](unsigned long long tile) {
    mbar_arrive_expect_tx(bar + B_VF + j, 8192);
    bulk_g2s(smem + CG_SV + j * 12288, args.ws + args.wl.off_v + tile * 8192, 8192, bar + B_VF + j);
  };
  // this warp is done reading the tri-bias stage of step (ii, kt); the last of the CTA's 8 warps refills
  // that stage with step + NB
  auto release_bias = [&](int ii, int kt) {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      const int bs = (ii * NT + kt) % CG_NB;
      if (atomicAdd(bias_cnt + bs, 1) == CG_SOFTMAX_WARPS - 1) {
        bias_cnt[bs] = 0;
        fence_proxy_async_smem();
        int i3 = ii, k3 = kt + CG_NB;
        while (k3 >= NT) { k3 -= NT; ++i3; }
        load_bias(i3, k3, ii);
      }
    }
    __syncwarp();
  };

  // the class word of the item two ahead, prefetched by the row's quad-0 warp (lane l: kt = 4l..4l+3)
  uint32_t cls_pf = quad == 0 ? class_word(blockIdx.x + gridDim.x, j, lane) : 0u;
  // first item: Q, K, V of the row's first active tile
  if (leader) {
    const int k0 = next_active(0, 0);
    if (k0 < NT) {
      const unsigned long long tb = tile_base(blockIdx.x);
      load_q(tb + core_item(blockIdx.x, NT, G).qt);
      load_k(tb + k0);
      load_v(tb + k0);
    }
  }
  int n = 0;   // active tiles processed by this row (all items): phase of KF/VF/SF/OF
  int nq = 0;  // Q tiles consumed by this row: phase of QF (leader only)
  int ii = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++ii) {
    const int cs = ii & 1;
    // classes of the next item into slot cs ^ 1 (its last readers, item ii - 1, finished before the
    // item barrier), then start loading those of the item after it
    if (quad == 0) {
      reinterpret_cast<uint32_t*>(scls + ((cs ^ 1) * CG_RG + j) * TILE)[lane] = cls_pf;
      cls_pf = class_word(item + 2 * gridDim.x, j, lane);
      __syncwarp();
    }
    if (leader) {
      const int first = next_active(cs, 0), nf = next_active(cs ^ 1, 0);
      rs->cur = tile_base(item);
      rs->nxt_first = nf;
      if (nf < NT) {
        rs->nxt = tile_base(item + gridDim.x);
        rs->nxt_qt = core_item(item + gridDim.x, NT, G).qt;
      }
      // a row without active tiles in this item fetches the next item's first tiles now
      if (first == NT && nf < NT) {
        load_q(rs->nxt + rs->nxt_qt);
        load_k(rs->nxt + nf);
        load_v(rs->nxt + nf);
      }
      if (first < NT) {
        mbar_wait(bar + B_QF + j, nq & 1, status, DEV_TIMEOUT_TMA);
        ++nq;
      }
    }

    float o[C_HEAD], l = 0.f, m = 0.f;
    bool started = false;
#pragma unroll
    for (int d = 0; d < C_HEAD; ++d) o[d] = 0.f;
    const uint8_t* my_cls = scls + (cs * CG_RG + j) * TILE;

    for (int kt = 0; kt < NT; ++kt) {
      const int s = ii * NT + kt;  // step of the CTA's bias ring
      const int bs = s % CG_NB;
      const int cls = my_cls[kt];
      const bool act = cls == 0 || cls == 2;
      float alpha = 1.f;
      if (act && leader) {
        // S = Q K^T + tri bias: the bias block [k/8][q][8] is a K-major fp16 operand (LBO 2048 B, SBO 128 B);
        // against the 64 x 64 identity it adds bias[q][k] to column k of S exactly, one 64-key half at a time
        mbar_wait(bar + B_KF + j, n & 1, status, DEV_TIMEOUT_TMA);
        mbar_wait(bar + B_BF + bs, (s / CG_NB) & 1, status, DEV_TIMEOUT_TMA);
        tc_fence_after();
#pragma unroll
        for (int k2 = 0; k2 < C_HEAD / 16; ++k2) {
          const uint64_t ad = smem_desc_noswizzle(smem_u32(smem + CG_SQ + j * 8192) + k2 * 256, 128, 512);
          const uint64_t bd = smem_desc_noswizzle(smem_u32(smem + CG_SK + j * 8192) + k2 * 256, 128, 512);
          umma_ss(buf0, ad, bd, idS, k2 > 0 ? 1u : 0u);
        }
        const uint32_t sbb = smem_u32(smem + CG_SB + bs * 32768), sid = smem_u32(smem + CG_SI);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint64_t ad = smem_desc_noswizzle(sbb + (8 * kh + 2 * k4) * 2048, 2048, 128);
            const uint64_t bd = smem_desc_noswizzle(sid + 256 * k4, 128, 1024);
            umma_ss(buf0 + 64 * kh, ad, bd, idB, 1u);
          }
        }
        umma_commit(bar + B_SF + j);
      }
      mbar_wait(bar + B_BF + bs, (s / CG_NB) & 1, status, DEV_TIMEOUT_TMA);
      if (act) {
        mbar_wait(bar + B_SF + j, n & 1, status, DEV_TIMEOUT_MMA);
        __syncwarp();
        tc_fence_after();
        if (leader) {  // S has consumed the K slot (and, after the row's last tile, the Q slot)
          const int kn = next_active(cs, kt + 1);
          if (kn < NT) {
            load_k(rs->cur + kn);
          } else if (rs->nxt_first < NT) {
            load_q(rs->nxt + rs->nxt_qt);
            load_k(rs->nxt + rs->nxt_first);
          }
        }
        const float* mbp = reinterpret_cast<const float*>(smem + CG_SMB + (bs * CG_RG + j) * 512);
        // pass 1: x = S (tri bias included by the MMA) (+ mask bias, written back over S), row max
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t sr[32];
          tmem_ld32(buf + 32 * c, sr);
          tmem_ld_wait();
          tmem_regs_ready(sr);
          float xs[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) xs[i] = __uint_as_float(sr[i]);
          if (cls == 2) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 mv = *reinterpret_cast<const float4*>(mbp + 32 * c + i);
              xs[i] += mv.x; xs[i + 1] += mv.y; xs[i + 2] += mv.z; xs[i + 3] += mv.w;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            mxa = max3f(mxa, xs[i], xs[i + 1]);
            mxb = max3f(mxb, xs[i + 2], xs[i + 3]);
            mxc = max3f(mxc, xs[i + 4], xs[i + 5]);
            mxd = max3f(mxd, xs[i + 6], xs[i + 7]);
          }
          if (cls == 2) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sr[i] = __float_as_uint(xs[i]);
            tmem_st32(buf + 32 * c, sr);
          }
        }
        tmem_st_wait();
        release_bias(ii, kt);
        const float mx = fmaxf(max3f(mxa, mxb, mxc), mxd);
        // lazy rescale: keep the running maximum unless it grew by more than 8 (a factor 256)
        if (!started) {
          m = mx;
          started = true;
        } else if (mx > m + 8.0f) {
          alpha = ex2(m - mx);
          m = mx;
        }
        const uint32_t nm = __float_as_uint(-m);
        const uint64_t neg_m2 = ((uint64_t)nm << 32) | nm;
        // pass 2: P = 2^(x - m) as fp16 pairs into columns [0, 64)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t xr[32];
          tmem_ld32(buf + 32 * c, xr);
          tmem_ld_wait();
          tmem_regs_ready(xr);
          uint32_t pk[16];
          // 10 of every 16 pairs on the MUFU, 6 on the FMA/ALU pipes (the split that balances the two)
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = (i % 8) < 5 ? exp2_pair_f16(__uint_as_float(xr[2 * i]), __uint_as_float(xr[2 * i + 1]), neg_m2)
                                : exp2_pair_poly_f16(__uint_as_float(xr[2 * i]), __uint_as_float(xr[2 * i + 1]), neg_m2);
          tmem_st16(buf + 16 * c, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        wg_sync(j);  // every warp of the row has stored its P
        if (leader) {
          tc_fence_after();
          mbar_wait(bar + B_VF + j, n & 1, status, DEV_TIMEOUT_TMA);
#pragma unroll
          for (int i = 0; i < TILE / 16; ++i) {
            const uint64_t bd = smem_desc_noswizzle(smem_u32(smem + CG_SV + j * 12288) + i * 256, 128, 2048);
            umma_ts(buf0 + 64, buf0 + i * 8, bd, idPV, i > 0 ? 1u : 0u);
          }
          umma_commit(bar + B_OF + j);
        }
        mbar_wait(bar + B_OF + j, n & 1, status, DEV_TIMEOUT_MMA);
        __syncwarp();
        tc_fence_after();
        if (leader) {  // P.V has consumed the V slot
          const int kn = next_active(cs, kt + 1);
          if (kn < NT) load_v(rs->cur + kn);
          else if (rs->nxt_first < NT) load_v(rs->nxt + rs->nxt_first);
        }
        uint32_t ov[32], lv[16];
        tmem_ld32(buf + 64, ov);
        tmem_ld16(buf + 96, lv);
        tmem_ld_wait();
        tmem_regs_ready(ov);
        tmem_regs_ready(lv);
#pragma unroll
        for (int d = 0; d < C_HEAD; ++d) o[d] = fmaf(o[d], alpha, __uint_as_float(ov[d]));
        l = fmaf(l, alpha, __uint_as_float(lv[0]));
        tc_fence_before();
        wg_sync(j);  // the row's columns are free for the next S
        ++n;
      } else {
        release_bias(ii, kt);
      }
    }

    // ---- epilogue: o / l -> fp16 core image of (b, row, qt), channels h*32.. (the sigmoid gate is
    //      applied by the output projection, which streams the matching g tile) ----
    if (started) {
      const CoreItem ci = core_item(item, NT, G);
      const int q = ci.qt * TILE + t;
      const bool qvalid = q < N;
      const float inv_l = 1.0f / l;
      unsigned char* cimg = args.ws + args.wl.off_core + (((size_t)ci.b * R + ci.g0 + j) * NT + ci.qt) * 32768;
#pragma unroll
      for (int d = 0; d < C_HEAD; d += 8) {
        uint32_t ow[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          ow[i] = qvalid ? H16<__half>::pack(o[d + 2 * i] * inv_l, o[d + 2 * i + 1] * inv_l) : 0u;
        *reinterpret_cast<uint4*>(cimg + img_off(t, ci.h * C_HEAD + d, HC)) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
    // bias addressing of item ii + 2 (its slot last served item ii - 1, whose refills are all done)
    if (tid == 0) iinfo[(ii + 2) % 3] = item_info(item + 2 * gridDim.x);
    __syncthreads();  // item barrier: class slot cs and item-info slot ii % 3 are free again
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, CG_RG * 128);
}

template <typename T>
static cudaError_t core_tc_launch(const LayerArgs& a, cudaStream_t st) {
  cudaFuncSetAttribute(core_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, CG_SMEM);
  const int R = a.row_end - a.row_begin;
  const int n_items = a.wl.NT * ((R + CG_RG - 1) / CG_RG) * a.B * HEADS;
  const int grid = n_items < 2 * a.num_sms ? n_items : 2 * a.num_sms;  // two resident CTAs per SM
  core_tc_kernel<T><<<grid, CG_THREADS, CG_SMEM, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_core_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  return dtype == DT_BF16 ? core_tc_launch<__nv_bfloat16>(a, st) : core_tc_launch<__half>(a, st);
}

// =================================================================================================
// Output projection (+ residual, optionally + the next module's LayerNorm).  Tile = 128 pairs (one
// query tile of one attention row): y[128 x 128] = (core o sigmoid(g))[128 x 128] * W_o^T, 256 threads.
// The CTA loops over tiles.  Output blocks in peer GPUs' memory: a persistent grid of three CTAs per
// SM, so the system-scope fence that publishes the remote stores runs once per CTA at the very end
// and the stores drain while the next tiles are computed (a fence per tile held every CTA slot until
// its 64 KB had crossed NVLink).  Local output: one tile per CTA, which the hardware's dynamic CTA
// scheduling balances better than a static tile split.
//   gate: warp w updates rows 16w..16w+15 of the core image; one warp instruction covers 8 rows x 4
//     chunks of 8 channels (lane = row % 8 + 8 * (chunk % 4)): g is read in 64-byte runs of 8 rows and
//     the image in four conflict-free 128-byte runs.
//   epilogue: the accumulator is staged through shared memory (fp32 rows at a stride of 132 floats:
//     conflict-free both ways), then warp w streams rows 16w..16w+15 whole (lane = 4 channels): the
//     residual loads, the output stores and the next LayerNorm's 16-bit rows are full 512 / 256-byte
//     runs, and the LayerNorm statistics are warp reductions over one row.
// =================================================================================================
constexpr int OP_THREADS = 256;
constexpr int OP_STAGE_LD = C_IN + 4;                 // staged row stride (floats)
constexpr int OP_SMEM_BODY = TILE * OP_STAGE_LD * 4;  // 67584 B: covers the two 32 KB operand images
constexpr int OP_SMEM = OP_SMEM_BODY + 64;
static_assert(OP_SMEM_BODY >= 65536, "staging buffer overlays the operand images");

template <typename T, bool LN_NEXT, bool PERSIST, bool TB>
__global__ void __launch_bounds__(OP_THREADS, 3) out_proj_tc_kernel(LayerArgs args) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sA = smem;
  unsigned char* sW = smem + 32768;
  float* stage = reinterpret_cast<float*>(smem);  // after the MMA: [128][OP_STAGE_LD] fp32
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OP_SMEM_BODY);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = args.N, R = args.row_end - args.row_begin, NT = args.wl.NT;
  const int n_tiles = NT * R * args.B;
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
  auto run_tile = [&](const int tile, const uint32_t par) {
    const int ct = tile % NT, al = (tile / NT) % R, b = tile / (NT * R), a = args.row_begin + al;
    if (tid == 0) {
      mbar_arrive_expect_tx(bars + 0, 65536);
      bulk_g2s(sA, args.ws + args.wl.off_core + (((size_t)b * R + al) * NT + ct) * 32768, 32768, bars + 0);
      bulk_g2s(sW, args.packed + PackedLayout::img_o, 32768, bars + 0);
    }
    // the epilogue's residual rows pulled into L2 while the gate and the MMA run, where they are one
    // contiguous run (a dense view with consecutive pairs as columns)
    if (tid == 32 && args.add_residual && !args.zv.cblk && args.zv.s_col == C_IN) {
      const int rows = min(TILE, N - ct * TILE);
      prefetch_l2_bulk(args.z + b * args.zv.s_batch + (long long)(a - args.zv.row0) * args.zv.s_row +
                           (long long)ct * TILE * C_IN,
                       rows * C_IN * 4);
    }
    // ---- gate: the fp16 core image times sigmoid(g) of the same (b, row, query), rounded once to T, in
    //      place (the MMA then reads a T image); g loads in flight before the image lands ----
    {
      const int r8 = lane & 7, kq = lane >> 3;
      const unsigned char* gb = args.ws + args.wl.off_g + ((size_t)b * R + al) * N * C_IN * 2;
      uint4 gv[8];
  #pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = 16 * warp + 8 * (it >> 2) + r8, k = 4 * (it & 3) + kq;
        const int q = min(ct * TILE + r, N - 1);
        gv[it] = __ldcs(reinterpret_cast<const uint4*>(gb + ((size_t)q * C_IN + 8 * k) * 2));
      }
      mbar_wait(bars + 0, par, status, DEV_TIMEOUT_TMA);
  #pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = 16 * warp + 8 * (it >> 2) + r8, k = 4 * (it & 3) + kq;
        uint4* cp = reinterpret_cast<uint4*>(sA + img_off(r, 8 * k, HC));
        const uint4 cv = *cp;
        const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, gw[4] = {gv[it].x, gv[it].y, gv[it].z, gv[it].w};
        uint32_t ow[4];
  #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 c2 = H16<__half>::unpack(cw[e]);
          const float2 g2 = H16<T>::unpack(gw[e]);
          if constexpr (H16<T>::is_bf16) {
            // bf16: c sigmoid(g) = c (1 + tanh(g / 2)) / 2 with the one-instruction MUFU tanh (about 2^-12
            // absolute in the sigmoid, far below bf16's rounding of the product); one MUFU operation
            // per element instead of two
            float t0, t1;
            asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(0.5f * g2.x));
            asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(0.5f * g2.y));
            const float hx = 0.5f * c2.x, hy = 0.5f * c2.y;
            ow[e] = H16<T>::pack(fmaf(hx, t0, hx), fmaf(hy, t1, hy));
          } else {
            ow[e] = H16<T>::pack(__fdividef(c2.x, 1.0f + __expf(-g2.x)), __fdividef(c2.y, 1.0f + __expf(-g2.y)));
          }
        }
        *cp = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
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
    // ---- epilogue.  Warp w streams rows 16w..16w+15 (lane: channels 4 lane..+3); the residual of its
    //      first 8 rows is in flight during the CTA barrier that follows the staging (out may alias z:
    //      a row's residual is always read before that row is written, and rows belong to one warp) ----
    auto row_off = [&](const View& v, int r) -> long long {
      return b * v.s_batch + (long long)(a - v.row0) * v.s_row + view_col(v, ct * TILE + r);
    };
    float4 zz[8];
    auto load_z = [&](int h) {
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 16 * warp + 8 * h + i;
        zz[i] = (args.add_residual && ct * TILE + r < N)
                    ? __ldcs(reinterpret_cast<const float4*>(args.z + row_off(args.zv, r)) + lane)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    float4 lw = make_float4(0.f, 0.f, 0.f, 0.f), lb = lw;
    if constexpr (LN_NEXT) {
      lw = __ldg(reinterpret_cast<const float4*>(args.ln_next_w) + lane);
      lb = __ldg(reinterpret_cast<const float4*>(args.ln_next_b) + lane);
    }
    mbar_wait(bars + 1, par, status, DEV_TIMEOUT_MMA);  // MMA done: the operand images are free for staging
    __syncwarp();
    tc_fence_after();
    {
      // TMEM -> stage: warp (quad, part) holds rows 32 quad.. (its lanes), columns 64 part..
      const int quad = warp & 3, part = warp >> 2;
      float* srow = stage + (quad * 32 + lane) * OP_STAGE_LD + 64 * part;
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
    load_z(0);
    tc_fence_before();
    __syncthreads();
    // the next tri bias from the rounded LayerNorm rows (kernel-uniform): lane 8 hh + i keeps head hh of
    // rows 16 warp + i (tbk0) and 16 warp + 8 + i (tbk1), stored once the warp's 16 rows are done
    constexpr bool tb_out = LN_NEXT && TB;
    float tbk0 = 0.f, tbk1 = 0.f;
  #pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      if (h == 1) load_z(1);
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 16 * warp + 8 * h + i;
        if (ct * TILE + r >= N) continue;  // warp-uniform
        const float4 s = *reinterpret_cast<const float4*>(stage + r * OP_STAGE_LD + 4 * lane);
        const float4 y = make_float4(s.x + zz[i].x, s.y + zz[i].y, s.z + zz[i].z, s.w + zz[i].w);
        __stcs(reinterpret_cast<float4*>(args.out + row_off(args.ov, r)) + lane, y);
        if constexpr (LN_NEXT) {
          // the next module's LayerNorm of the new row (reference linear_addln, kernels_nax3.py:69-198):
          // two-pass fp32 statistics, one rounding to the 16-bit type
          const float mean = warp_sum32((y.x + y.y) + (y.z + y.w)) * (1.0f / C_IN);
          const float d0 = y.x - mean, d1 = y.y - mean, d2 = y.z - mean, d3 = y.w - mean;
          const float var = warp_sum32((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3)) * (1.0f / C_IN);
          const float rstd = rsqrtf(var + LN_EPS);
          uint2 pk;
          pk.x = H16<T>::pack(d0 * rstd * lw.x + lb.x, d1 * rstd * lw.y + lb.y);
          pk.y = H16<T>::pack(d2 * rstd * lw.z + lb.z, d3 * rstd * lw.w + lb.w);
          *(reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(args.ln_out) + row_off(args.lnv, r)) + lane) = pk;
          if constexpr (tb_out) {
            // reference _LN_EPI_TB (kernels_nax3.py:104-143): fp32 sums of the rounded LayerNorm values
            const float2 a01 = H16<T>::unpack(pk.x), a23 = H16<T>::unpack(pk.y);
            float p[HEADS];
  #pragma unroll
            for (int hh = 0; hh < HEADS; ++hh) {
              const float4 w = __ldg(reinterpret_cast<const float4*>(args.tb_next_w + hh * C_IN) + lane);
              p[hh] = a01.x * w.x + a01.y * w.y + a23.x * w.z + a23.y * w.w;
            }
            const float k = head_sums4(p, lane);
            if ((lane & 7) == i) {
              if (h == 0) tbk0 = k;
              else tbk1 = k;
            }
          }
        }
      }
    }
    if constexpr (tb_out) {
      // fp16 [B][HEADS][N][N], the pair index of ln_out (a dense view: row0 = 0, no block table)
      const int i = lane & 7, hh = lane >> 3;
  #pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = 16 * warp + 8 * h + i;
        if (ct * TILE + r < N) {
          const long long pidx = (row_off(args.lnv, r) - b * args.lnv.s_batch) / C_IN;
          reinterpret_cast<__half*>(args.tb_next)[((long long)b * HEADS + hh) * N * N + pidx] =
              __float2half_rn(h ? tbk1 : tbk0);
        }
      }
    }
    // the staging rows were read through the generic proxy; the next tile's bulk copies overwrite them
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
  };
  if constexpr (PERSIST) {
#pragma unroll 1
    for (int tile = blockIdx.x, iter = 0; tile < n_tiles; tile += gridDim.x, ++iter) run_tile(tile, iter & 1);
  } else {
    run_tile(blockIdx.x, 0);
  }
  // peer stores (output blocks in other GPUs' memory): performed system-wide before the kernel ends,
  // ahead of the cross-GPU barrier that publishes them
  if (args.ov.tab || args.lnv.tab) __threadfence_system();
  if (warp == 0) tmem_dealloc(tbase, 128);
}

template <typename T, bool LN_NEXT, bool TB = false>
static cudaError_t out_proj_tc_launch(const LayerArgs& a, cudaStream_t st) {
  const int n_tiles = a.wl.NT * (a.row_end - a.row_begin) * a.B;
  if (a.ov.tab || a.lnv.tab) {  // output blocks on peer GPUs: persistent, three resident CTAs per SM
    cudaFuncSetAttribute(out_proj_tc_kernel<T, LN_NEXT, true, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, OP_SMEM);
    const int grid = n_tiles < 3 * a.num_sms ? n_tiles : 3 * a.num_sms;
    out_proj_tc_kernel<T, LN_NEXT, true, TB><<<grid, OP_THREADS, OP_SMEM, st>>>(a);
  } else {
    cudaFuncSetAttribute(out_proj_tc_kernel<T, LN_NEXT, false, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, OP_SMEM);
    out_proj_tc_kernel<T, LN_NEXT, false, TB><<<n_tiles, OP_THREADS, OP_SMEM, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_out_proj_tc(const LayerArgs& a, int dtype, cudaStream_t st) {
  if (a.ln_out && a.tb_next)
    return dtype == DT_BF16 ? out_proj_tc_launch<__nv_bfloat16, true, true>(a, st)
                            : out_proj_tc_launch<__half, true, true>(a, st);
  if (a.ln_out)
    return dtype == DT_BF16 ? out_proj_tc_launch<__nv_bfloat16, true>(a, st) : out_proj_tc_launch<__half, true>(a, st);
  return dtype == DT_BF16 ? out_proj_tc_launch<__nv_bfloat16, false>(a, st) : out_proj_tc_launch<__half, false>(a, st);
}

}  // namespace triattn
