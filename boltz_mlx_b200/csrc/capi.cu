// extern "C" entry points of libtriattn.so (declared in include/triattn.h): host-side argument
// validation, workspace layout, stage dispatch on the caller's stream, device status word.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "triattn.h"
#include "triattn_internal.cuh"

namespace triattn {

__device__ int g_device_status = 0;

// Device address of the status word, resolved once per device (the __device__ variable has one
// instance per device that loads the library).
int* device_status_ptr() {
  static int* cache[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_device_status) != cudaSuccess) return nullptr;
    cache[dev] = p;
  }
  return cache[dev];
}

// Multiprocessor count of the current device, resolved once per device.
int device_sm_count() {
  static int cache[64] = {0};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 1;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace triattn

using namespace triattn;

namespace {

thread_local char g_err[512] = "";

}  // namespace

// Record a host-side error (read back by triattn_last_error_string) and return its code.
int triattn::record_error(int code, const char* what, const char* detail) {
  snprintf(g_err, sizeof(g_err), "%s: %s", what, detail);
  return code;
}

namespace {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TRIATTN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_dims(int B, int N, int dtype) {
  if (B < 1 || N < 1) return fail(TRIATTN_EINVAL, "B=%d N=%d must be >= 1", B, N);
  if (N > 16384) return fail(TRIATTN_EUNSUPPORTED, "N=%d above the supported 16384", N);
  if ((long long)B * HEADS > 65535) return fail(TRIATTN_EUNSUPPORTED, "B=%d too large", B);
  if (dtype != DT_F32 && dtype != DT_F16 && dtype != DT_BF16) return fail(TRIATTN_EUNSUPPORTED, "dtype %d", dtype);
  return TRIATTN_OK;
}

int check_rows(int N, int row_begin, int row_end) {
  if (row_begin < 0 || row_end > N || row_begin >= row_end)
    return fail(TRIATTN_EINVAL, "row range [%d,%d) outside [0,%d)", row_begin, row_end, N);
  if (row_end - row_begin > 65535) return fail(TRIATTN_EUNSUPPORTED, "row range longer than 65535");
  return TRIATTN_OK;
}

int check_ws(void* ws, size_t ws_bytes, const Workspace& wl) {
  if (!ws) return fail(TRIATTN_EINVAL, "workspace is NULL");
  if (!aligned(ws, 256)) return fail(TRIATTN_EINVAL, "workspace must be 256-byte aligned");
  if (ws_bytes < wl.total) return fail(TRIATTN_ENOSPACE, "workspace %zu bytes < %zu needed", ws_bytes, wl.total);
  return TRIATTN_OK;
}

int check_packed(const void* packed, int dtype) {
  if (!packed) return fail(TRIATTN_EINVAL, "packed weights are NULL");
  if (!aligned(packed, 256)) return fail(TRIATTN_EINVAL, "packed weights must be 256-byte aligned");
  (void)dtype;
  return TRIATTN_OK;
}

View pair_view(int N, int starting, int channels) {
  View v;
  v.s_batch = (long long)N * N * channels;
  v.s_row = starting ? (long long)N * channels : channels;
  v.s_col = starting ? channels : (long long)N * channels;
  v.row0 = 0;
  v.cblk = 0;
  v.s_cblk = 0;
  v.tab = nullptr;
  return v;
}

LayerArgs make_args(int B, int N, int starting, int row_begin, int row_end, float inf, const float* z,
                    const float* mask, float* out, int add_residual, const void* packed, void* ws, int dtype) {
  LayerArgs a{};
  a.B = B; a.N = N; a.row_begin = row_begin; a.row_end = row_end; a.inf = inf;
  a.z = z; a.zv = pair_view(N, starting, C_IN);
  a.mask = mask; a.mv = pair_view(N, starting, 1);
  a.out = out; a.ov = pair_view(N, starting, C_IN);
  a.add_residual = add_residual;
  a.packed = static_cast<const unsigned char*>(packed);
  a.ws = static_cast<unsigned char*>(ws);
  a.wl = Workspace::make(B, N, row_end - row_begin, dtype);
  a.status = device_status_ptr();
  a.num_sms = device_sm_count();
  a.xn = nullptr;
  a.ln_next_w = a.ln_next_b = nullptr;
  a.ln_out = nullptr;
  a.tb_in = nullptr;
  a.tb_next_w = nullptr;
  a.tb_next = nullptr;
  return a;
}

int finish(cudaError_t e, const char* what) { return e == cudaSuccess ? TRIATTN_OK : cuda_fail(e, what); }

}  // namespace

extern "C" {

const char* triattn_version(void) { return "triattn-b200 0.1 (sm_100a)"; }

const char* triattn_last_error_string(void) { return g_err; }

int triattn_device_status(int* status, int clear) {
  if (!status) return fail(TRIATTN_EINVAL, "status is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol");
  *status = v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol");
  }
  return TRIATTN_OK;
}

size_t triattn_packed_weights_bytes(int dtype) { return PackedLayout::bytes(dtype); }

int triattn_pack_weights(const float* ln_w, const float* ln_b, const float* w_q, const float* w_k, const float* w_v,
                         const float* w_g, const float* g_bias, const float* w_b, const float* w_o, int dtype,
                         void* packed, size_t packed_bytes, void* stream) {
  if (dtype != DT_F32 && dtype != DT_F16 && dtype != DT_BF16) return fail(TRIATTN_EUNSUPPORTED, "dtype %d", dtype);
  if (!ln_w || !ln_b || !w_q || !w_k || !w_v || !w_g || !w_b || !w_o)
    return fail(TRIATTN_EINVAL, "a weight pointer is NULL");
  if (int r = check_packed(packed, dtype)) return r;
  if (packed_bytes < PackedLayout::bytes(dtype))
    return fail(TRIATTN_ENOSPACE, "packed buffer %zu < %zu bytes", packed_bytes, PackedLayout::bytes(dtype));
  return finish(launch_pack_weights(ln_w, ln_b, w_q, w_k, w_v, w_g, g_bias, w_b, w_o, dtype,
                                    static_cast<unsigned char*>(packed), static_cast<cudaStream_t>(stream)),
                "pack_weights");
}

size_t triattn_workspace_bytes(int B, int N, int rows, int dtype) {
  if (B < 1 || N < 1 || rows < 1) return 0;
  return Workspace::make(B, N, rows, dtype).total;
}

int triattn_mask_prep(const float* mask, int B, int N, int starting, float inf, int row_begin, int row_end,
                      int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  LayerArgs a = make_args(B, N, starting, row_begin, row_end, inf, nullptr, mask, nullptr, 0, nullptr, workspace, dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  return finish(launch_mask_prep(a, dtype, static_cast<cudaStream_t>(stream)), "mask_prep");
}

int triattn_ln_proj(const float* z, const void* packed, int B, int N, int starting, int row_begin, int row_end,
                    int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  if (!z || !aligned(z, 16)) return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer");
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, starting, row_begin, row_end, 0.f, z, nullptr, nullptr, 0, packed, workspace, dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return finish(dtype == DT_F32 ? launch_ln_proj_f32(a, st) : launch_ln_proj_tc(a, dtype, st), "ln_proj");
}

int triattn_core(int B, int N, int row_begin, int row_end, int dtype, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  LayerArgs a = make_args(B, N, 1, row_begin, row_end, 0.f, nullptr, nullptr, nullptr, 0, nullptr, workspace, dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return finish(dtype == DT_F32 ? launch_core_f32(a, st) : launch_core_tc(a, dtype, st), "core");
}

int triattn_out_proj(const float* z, const void* packed, int B, int N, int starting, int row_begin, int row_end,
                     int dtype, int add_residual, float* out, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  if (!out || !aligned(out, 16)) return fail(TRIATTN_EINVAL, "out must be a 16-byte aligned device pointer");
  if (add_residual && (!z || !aligned(z, 16))) return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer");
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, starting, row_begin, row_end, 0.f, z, nullptr, out, add_residual, packed, workspace,
                          dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return finish(dtype == DT_F32 ? launch_out_proj_f32(a, st) : launch_out_proj_tc(a, dtype, st), "out_proj");
}

static int check_view(const char* name, const void* p, int64_t sb, int64_t sr, int64_t sc, bool vec4) {
  if (!p) return fail(TRIATTN_EINVAL, "%s is NULL", name);
  if (sb < 0 || sr < 0 || sc < 0) return fail(TRIATTN_EINVAL, "%s: negative stride", name);
  if (vec4 && (!aligned(p, 16) || sb % 4 || sr % 4 || sc % 4))
    return fail(TRIATTN_EINVAL, "%s: base must be 16-byte aligned and strides multiples of 4 elements", name);
  return TRIATTN_OK;
}

static View make_view(int64_t sb, int64_t sr, int64_t sc, int row0, int cblk = 0, int64_t s_cblk = 0) {
  View v;
  v.s_batch = sb; v.s_row = sr; v.s_col = sc; v.row0 = row0;
  v.cblk = cblk; v.s_cblk = s_cblk;
  v.tab = nullptr;
  return v;
}

static int check_blocks(const char* name, int N, int cblk, int64_t s_cblk) {
  if (cblk < 0 || (cblk > 0 && (N % cblk || s_cblk < 0 || s_cblk % 4)))
    return fail(TRIATTN_EINVAL, "%s: column blocks must divide N, with a non-negative stride of whole 16-byte rows", name);
  return TRIATTN_OK;
}

int triattn_mask_prep_v(const float* mask, int64_t s_batch, int64_t s_row, int64_t s_col, int B, int N, float inf,
                        int row_begin, int row_end, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  if (mask && s_batch < 0) return fail(TRIATTN_EINVAL, "mask: negative stride");
  LayerArgs a = make_args(B, N, 1, row_begin, row_end, inf, nullptr, mask, nullptr, 0, nullptr, workspace, dtype);
  a.mv = make_view(s_batch, s_row, s_col, row_begin);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  return finish(launch_mask_prep(a, dtype, static_cast<cudaStream_t>(stream)), "mask_prep_v");
}

int triattn_ln_proj_v(const float* z, int64_t s_batch, int64_t s_row, int64_t s_col, const void* packed, int B, int N,
                      int row_begin, int row_end, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return triattn_ln_proj_vb(z, s_batch, s_row, s_col, 0, 0, packed, B, N, row_begin, row_end, dtype, workspace,
                            workspace_bytes, stream);
}

int triattn_ln_proj_vb(const float* z, int64_t s_batch, int64_t s_row, int64_t s_col, int col_block, int64_t s_col_block,
                       const void* packed, int B, int N, int row_begin, int row_end, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  if (int r = check_view("z", z, s_batch, s_row, s_col, true)) return r;
  if (int r = check_blocks("z", N, col_block, s_col_block)) return r;
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, 1, row_begin, row_end, 0.f, z, nullptr, nullptr, 0, packed, workspace, dtype);
  a.zv = make_view(s_batch, s_row, s_col, row_begin, col_block, s_col_block);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return finish(dtype == DT_F32 ? launch_ln_proj_f32(a, st) : launch_ln_proj_tc(a, dtype, st), "ln_proj_v");
}

int triattn_out_proj_v(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col, float* out,
                       int64_t os_batch, int64_t os_row, int64_t os_col, const void* packed, int B, int N,
                       int row_begin, int row_end, int dtype, int add_residual, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return triattn_out_proj_vb(z, zs_batch, zs_row, zs_col, 0, 0, out, os_batch, os_row, os_col, 0, 0, packed, B, N,
                             row_begin, row_end, dtype, add_residual, workspace, workspace_bytes, stream);
}

static int out_proj_blocks(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col, int z_col_block,
                           int64_t zs_col_block, float* out, int64_t os_batch, int64_t os_row, int64_t os_col,
                           int o_col_block, int64_t os_col_block, const int64_t* o_block_table, const void* packed,
                           int B, int N, int row_begin, int row_end, int dtype, int add_residual, void* workspace,
                           size_t workspace_bytes, void* stream, const char* what) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (int r = check_rows(N, row_begin, row_end)) return r;
  if (int r = check_view("out", out, os_batch, os_row, os_col, true)) return r;
  if (int r = check_blocks("out", N, o_col_block, os_col_block)) return r;
  if (o_block_table && (o_col_block <= 0 || !aligned(o_block_table, 8)))
    return fail(TRIATTN_EINVAL, "out: a block table needs column blocks and 8-byte alignment");
  if (add_residual) {
    if (int r = check_view("z", z, zs_batch, zs_row, zs_col, true)) return r;
    if (int r = check_blocks("z", N, z_col_block, zs_col_block)) return r;
  }
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, 1, row_begin, row_end, 0.f, z, nullptr, out, add_residual, packed, workspace, dtype);
  a.zv = make_view(zs_batch, zs_row, zs_col, row_begin, z_col_block, zs_col_block);
  a.ov = make_view(os_batch, os_row, os_col, row_begin, o_col_block, os_col_block);
  a.ov.tab = reinterpret_cast<const long long*>(o_block_table);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_EINVAL, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return finish(dtype == DT_F32 ? launch_out_proj_f32(a, st) : launch_out_proj_tc(a, dtype, st), what);
}

int triattn_out_proj_vb(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col, int z_col_block,
                        int64_t zs_col_block, float* out, int64_t os_batch, int64_t os_row, int64_t os_col,
                        int o_col_block, int64_t os_col_block, const void* packed, int B, int N, int row_begin,
                        int row_end, int dtype, int add_residual, void* workspace, size_t workspace_bytes,
                        void* stream) {
  return out_proj_blocks(z, zs_batch, zs_row, zs_col, z_col_block, zs_col_block, out, os_batch, os_row, os_col,
                         o_col_block, os_col_block, nullptr, packed, B, N, row_begin, row_end, dtype, add_residual,
                         workspace, workspace_bytes, stream, "out_proj_v");
}

int triattn_out_proj_vt(const float* z, int64_t zs_batch, int64_t zs_row, int64_t zs_col, int z_col_block,
                        int64_t zs_col_block, float* out, int64_t os_batch, int64_t os_row, int64_t os_col,
                        int o_col_block, const int64_t* o_block_table, const void* packed, int B, int N,
                        int row_begin, int row_end, int dtype, int add_residual, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!o_block_table) return fail(TRIATTN_EINVAL, "out: block table is NULL");
  return out_proj_blocks(z, zs_batch, zs_row, zs_col, z_col_block, zs_col_block, out, os_batch, os_row, os_col,
                         o_col_block, 0, o_block_table, packed, B, N, row_begin, row_end, dtype, add_residual,
                         workspace, workspace_bytes, stream, "out_proj_vt");
}

// ---- peer-store exchange: IPC-shareable buffers and the cross-GPU barrier ----------------------
int triattn_peer_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return fail(TRIATTN_EINVAL, "peer_alloc: NULL result pointer or zero size");
  *dev_ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (peer buffer)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaMemset (peer buffer)");
  }
  *dev_ptr = p;
  return TRIATTN_OK;
}

int triattn_peer_free(void* dev_ptr) {
  if (!dev_ptr) return TRIATTN_OK;
  return finish(cudaFree(dev_ptr), "cudaFree (peer buffer)");
}

int triattn_ipc_handle(void* dev_ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == TRIATTN_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle) return fail(TRIATTN_EINVAL, "ipc_handle: NULL pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return TRIATTN_OK;
}

int triattn_ipc_open(const void* handle, void** dev_ptr) {
  if (!dev_ptr || !handle) return fail(TRIATTN_EINVAL, "ipc_open: NULL pointer");
  *dev_ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return finish(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int triattn_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return TRIATTN_OK;
  return finish(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

int triattn_peer_broadcast(const uint64_t* buf_ptrs, int rank, int world, size_t offset, size_t bytes,
                           void* stream) {
  if (!buf_ptrs || !aligned(buf_ptrs, 8)) return fail(TRIATTN_EINVAL, "peer_broadcast: pointer table NULL or unaligned");
  if (world < 1 || world > 32 || rank < 0 || rank >= world)
    return fail(TRIATTN_EINVAL, "peer_broadcast: rank %d of %d (1..32 ranks)", rank, world);
  if (offset % 16 || bytes % 16) return fail(TRIATTN_EINVAL, "peer_broadcast: offset and size must be multiples of 16");
  return finish(launch_peer_broadcast(reinterpret_cast<const unsigned long long*>(buf_ptrs), rank, world, offset, bytes,
                                      device_sm_count(), static_cast<cudaStream_t>(stream)),
                "peer_broadcast");
}

int triattn_peer_barrier(const uint64_t* flag_ptrs, int rank, int world, uint32_t epoch, void* stream) {
  if (!flag_ptrs || !aligned(flag_ptrs, 8)) return fail(TRIATTN_EINVAL, "peer_barrier: flag table NULL or unaligned");
  if (world < 1 || world > 32 || rank < 0 || rank >= world)
    return fail(TRIATTN_EINVAL, "peer_barrier: rank %d of %d (1..32 ranks)", rank, world);
  int* status = device_status_ptr();
  if (!status) return fail(TRIATTN_EINVAL, "device status word unavailable");
  return finish(launch_peer_barrier(reinterpret_cast<const unsigned long long*>(flag_ptrs), rank, world, epoch, status,
                                    static_cast<cudaStream_t>(stream)),
                "peer_barrier");
}

int triattn_forward_fused(const float* z, const void* xn, const float* mask, const void* packed, int B, int N,
                          int starting, float inf, int dtype, int add_residual, float* out, int out_attn_layout,
                          const float* ln_next_w, const float* ln_next_b, void* ln_out, int ln_out_swapped,
                          void* workspace, size_t workspace_bytes, void* stream) {
  return triattn_forward_fused_tb(z, xn, nullptr, mask, packed, B, N, starting, inf, dtype, add_residual, out,
                                  out_attn_layout, ln_next_w, ln_next_b, ln_out, ln_out_swapped, nullptr, nullptr,
                                  workspace, workspace_bytes, stream);
}

int triattn_forward_fused_tb(const float* z, const void* xn, const void* tb, const float* mask, const void* packed,
                             int B, int N, int starting, float inf, int dtype, int add_residual, float* out,
                             int out_attn_layout, const float* ln_next_w, const float* ln_next_b, void* ln_out,
                             int ln_out_swapped, const float* tb_next_w, void* tb_next, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (tb && !xn) return fail(TRIATTN_EINVAL, "tb (the producer's tri bias) comes with xn, the producer's LayerNorm output");
  if (tb && !aligned(tb, 2)) return fail(TRIATTN_EINVAL, "tb must be a 2-byte aligned device pointer");
  if (tb_next && (!ln_out || !tb_next_w || !aligned(tb_next, 2) || !aligned(tb_next_w, 16)))
    return fail(TRIATTN_EINVAL, "tb_next needs ln_out, a 16-byte aligned tb_next_w and a 2-byte aligned tb_next");
  if ((xn || ln_out) && dtype == DT_F32)
    return fail(TRIATTN_EUNSUPPORTED, "xn / ln_out belong to the 16-bit path (the reference's f16 pair block)");
  if (!out || !aligned(out, 16)) return fail(TRIATTN_EINVAL, "out must be a 16-byte aligned device pointer");
  if ((add_residual || !xn) && (!z || !aligned(z, 16)))
    return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer (residual or LayerNorm input)");
  if (xn && !aligned(xn, 16)) return fail(TRIATTN_EINVAL, "xn must be 16-byte aligned");
  if (ln_out && (!aligned(ln_out, 16) || !ln_next_w || !ln_next_b || !aligned(ln_next_w, 16) || !aligned(ln_next_b, 16)))
    return fail(TRIATTN_EINVAL, "ln_out needs 16-byte aligned ln_out, ln_next_w and ln_next_b");
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, starting, 0, N, inf, z, mask, out, add_residual, packed, workspace, dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  if (xn) {
    a.xn = xn;
    a.xnv = pair_view(N, 1, C_IN);  // the layer's attention orientation (ending node: already transposed)
  }
  if (out_attn_layout) a.ov = pair_view(N, 1, C_IN);
  if (ln_out) {
    a.ln_next_w = ln_next_w;
    a.ln_next_b = ln_next_b;
    a.ln_out = ln_out;
    // z's orientation seen from this layer, or with the two N axes swapped
    a.lnv = pair_view(N, ln_out_swapped ? !starting : starting, C_IN);
  }
  a.tb_in = tb;
  a.tb_next_w = tb_next_w;
  a.tb_next = tb_next;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_mask_prep(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "mask_prep");
  e = dtype == DT_F32 ? launch_ln_proj_f32(a, st) : launch_ln_proj_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "ln_proj");
  e = dtype == DT_F32 ? launch_core_f32(a, st) : launch_core_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "core");
  e = dtype == DT_F32 ? launch_out_proj_f32(a, st) : launch_out_proj_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "out_proj");
  return TRIATTN_OK;
}

int triattn_forward(const float* z, const float* mask, const void* packed, int B, int N, int starting, float inf,
                    int dtype, int add_residual, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (!z || !aligned(z, 16)) return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer");
  if (!out || !aligned(out, 16)) return fail(TRIATTN_EINVAL, "out must be a 16-byte aligned device pointer");
  if (int r = check_packed(packed, dtype)) return r;
  LayerArgs a = make_args(B, N, starting, 0, N, inf, z, mask, out, add_residual, packed, workspace, dtype);
  if (int r = check_ws(workspace, workspace_bytes, a.wl)) return r;
  if (!a.status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_mask_prep(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "mask_prep");
  e = dtype == DT_F32 ? launch_ln_proj_f32(a, st) : launch_ln_proj_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "ln_proj");
  e = dtype == DT_F32 ? launch_core_f32(a, st) : launch_core_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "core");
  e = dtype == DT_F32 ? launch_out_proj_f32(a, st) : launch_out_proj_tc(a, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "out_proj");
  return TRIATTN_OK;
}

// ---- triangle multiplication ---------------------------------------------------------------------
size_t triattn_trimul_packed_bytes(int dtype) { return TrimulPacked::bytes(dtype); }

size_t triattn_trimul_workspace_bytes(int B, int N, int dtype) {
  if (B < 1 || N < 1) return 0;
  return TrimulWorkspace::make(B, N, dtype).total;
}

int triattn_trimul_pack_weights(const float* in_w, const float* in_b, const float* p_in, const float* g_in,
                                const float* out_w, const float* out_b, const float* p_out, const float* g_out,
                                int dtype, void* packed, size_t packed_bytes, void* stream) {
  if (!in_w || !in_b || !p_in || !g_in || !out_w || !out_b || !p_out || !g_out)
    return fail(TRIATTN_EINVAL, "trimul_pack_weights: a parameter pointer is NULL");
  if (dtype != DT_F32 && dtype != DT_F16 && dtype != DT_BF16) return fail(TRIATTN_EUNSUPPORTED, "dtype %d", dtype);
  if (!packed || !aligned(packed, 256)) return fail(TRIATTN_EINVAL, "packed must be a 256-byte aligned device pointer");
  if (packed_bytes < TrimulPacked::bytes(dtype))
    return fail(TRIATTN_ENOSPACE, "packed %zu bytes < %zu needed", packed_bytes, TrimulPacked::bytes(dtype));
  if (!aligned(in_w, 16) || !aligned(in_b, 16) || !aligned(out_w, 16) || !aligned(out_b, 16))
    return fail(TRIATTN_EINVAL, "LayerNorm parameters must be 16-byte aligned");
  return finish(launch_trimul_pack(in_w, in_b, p_in, g_in, out_w, out_b, p_out, g_out, dtype,
                                   static_cast<unsigned char*>(packed), static_cast<cudaStream_t>(stream)),
                "trimul_pack_weights");
}

static int trimul_call(const float* z, const float* mask, const void* packed, int B, int N, int outgoing, int dtype,
                       int add_residual, float* out, const float* ln_next_w, const float* ln_next_b, void* ln_out,
                       const float* tb_next_w, void* tb_next, void* workspace, size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if ((long long)B * N * N > 2147483647LL) return fail(TRIATTN_EUNSUPPORTED, "B*N*N above 2^31 pairs");
  if (!z || !aligned(z, 16)) return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer");
  if (!out || !aligned(out, 16)) return fail(TRIATTN_EINVAL, "out must be a 16-byte aligned device pointer");
  if (int r = check_packed(packed, dtype)) return r;
  const TrimulWorkspace wl = TrimulWorkspace::make(B, N, dtype);
  if (!workspace || !aligned(workspace, 256)) return fail(TRIATTN_EINVAL, "workspace must be 256-byte aligned");
  if (workspace_bytes < wl.total)
    return fail(TRIATTN_ENOSPACE, "workspace %zu bytes < %zu needed", workspace_bytes, wl.total);
  TrimulArgs a{};
  a.z = z; a.mask = mask; a.packed = static_cast<const unsigned char*>(packed);
  a.B = B; a.N = N; a.outgoing = outgoing ? 1 : 0; a.dtype = dtype; a.add_residual = add_residual ? 1 : 0;
  a.out = out; a.ws = static_cast<unsigned char*>(workspace);
  a.ln_next_w = ln_next_w; a.ln_next_b = ln_next_b; a.ln_out = ln_out;
  a.tb_next_w = tb_next_w; a.tb_next = tb_next;
  int blas = 0;
  const char* stage = "";
  const cudaError_t e = launch_trimul(a, static_cast<cudaStream_t>(stream), &blas, &stage);
  if (blas) return fail(TRIATTN_ECUDA, "trimul %s: cuBLAS status %d", stage, blas);
  if (e != cudaSuccess) return fail(TRIATTN_ECUDA, "trimul %s: %s", stage, cudaGetErrorString(e));
  return TRIATTN_OK;
}

int triattn_trimul_forward(const float* z, const float* mask, const void* packed, int B, int N, int outgoing,
                           int dtype, int add_residual, float* out, void* workspace, size_t workspace_bytes,
                           void* stream) {
  return trimul_call(z, mask, packed, B, N, outgoing, dtype, add_residual, out, nullptr, nullptr, nullptr, nullptr,
                     nullptr, workspace, workspace_bytes, stream);
}

int triattn_trimul_forward_addln(const float* z, const float* mask, const void* packed, int B, int N, int outgoing,
                                 int dtype, float* out, const float* ln_next_w, const float* ln_next_b, void* ln_out,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  return triattn_trimul_forward_addln_tb(z, mask, packed, B, N, outgoing, dtype, out, ln_next_w, ln_next_b, ln_out,
                                         nullptr, nullptr, workspace, workspace_bytes, stream);
}

int triattn_trimul_forward_addln_tb(const float* z, const float* mask, const void* packed, int B, int N, int outgoing,
                                    int dtype, float* out, const float* ln_next_w, const float* ln_next_b,
                                    void* ln_out, const float* tb_next_w, void* tb_next, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (dtype == DT_F32) return fail(TRIATTN_EUNSUPPORTED, "trimul addln belongs to the 16-bit path");
  if (!ln_out || !aligned(ln_out, 16) || !ln_next_w || !ln_next_b || !aligned(ln_next_w, 16) ||
      !aligned(ln_next_b, 16))
    return fail(TRIATTN_EINVAL, "ln_out needs 16-byte aligned ln_out, ln_next_w and ln_next_b");
  if (tb_next && (!tb_next_w || !aligned(tb_next, 2) || !aligned(tb_next_w, 16)))
    return fail(TRIATTN_EINVAL, "tb_next needs a 16-byte aligned tb_next_w and a 2-byte aligned tb_next");
  return trimul_call(z, mask, packed, B, N, outgoing, dtype, 1, out, ln_next_w, ln_next_b, ln_out, tb_next_w, tb_next,
                     workspace, workspace_bytes, stream);
}

int triattn_forward_chunked(const float* z, const float* mask, const void* packed, int B, int N, int starting,
                            float inf, int dtype, int add_residual, float* out, int chunk_rows, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (int r = check_dims(B, N, dtype)) return r;
  if (!z || !aligned(z, 16)) return fail(TRIATTN_EINVAL, "z must be a 16-byte aligned device pointer");
  if (!out || !aligned(out, 16)) return fail(TRIATTN_EINVAL, "out must be a 16-byte aligned device pointer");
  if (int r = check_packed(packed, dtype)) return r;
  if (chunk_rows < 1) return fail(TRIATTN_EINVAL, "chunk_rows=%d must be >= 1", chunk_rows);
  const int C = chunk_rows < N ? chunk_rows : N;
  if (dtype != DT_F32 && C < N && C % TILE)
    return fail(TRIATTN_EINVAL, "16-bit chunks hold whole 128-row tri-bias blocks: chunk_rows=%d", chunk_rows);
  if (int r = check_ws(workspace, workspace_bytes, Workspace::make(B, N, C, dtype))) return r;
  int* status = device_status_ptr();
  if (!status) return fail(TRIATTN_ECUDA, "device status word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nch = (N + C - 1) / C;
  auto args_of = [&](int k) {
    const int r0 = k * C, r1 = r0 + C < N ? r0 + C : N;
    return make_args(B, N, starting, r0, r1, inf, z, mask, out, add_residual, packed, workspace, dtype);
  };
  auto ln_proj = [&](const LayerArgs& a) {
    return dtype == DT_F32 ? launch_ln_proj_f32(a, st) : launch_ln_proj_tc(a, dtype, st);
  };
  // pass 1: the tri-bias rows of every chunk (the bias region is shared by all row counts); each
  // chunk's q|k|v|g rows land in the per-row regions and are overwritten by the next chunk
  for (int k = 0; k < nch; ++k) {
    cudaError_t e = ln_proj(args_of(k));
    if (e != cudaSuccess) return cuda_fail(e, "ln_proj (tri-bias pass)");
  }
  // pass 2, last chunk first: its projections from pass 1 are still in the workspace.  With out == z
  // (in place) a chunk writes only its own attention rows (ending node: its columns of z), which no
  // later chunk reads.
  for (int k = nch - 1; k >= 0; --k) {
    const LayerArgs a = args_of(k);
    cudaError_t e = launch_mask_prep(a, dtype, st);
    if (e != cudaSuccess) return cuda_fail(e, "mask_prep");
    if (k != nch - 1) {
      e = ln_proj(a);
      if (e != cudaSuccess) return cuda_fail(e, "ln_proj");
    }
    e = dtype == DT_F32 ? launch_core_f32(a, st) : launch_core_tc(a, dtype, st);
    if (e != cudaSuccess) return cuda_fail(e, "core");
    e = dtype == DT_F32 ? launch_out_proj_f32(a, st) : launch_out_proj_tc(a, dtype, st);
    if (e != cudaSuccess) return cuda_fail(e, "out_proj");
  }
  return TRIATTN_OK;
}

}  // extern "C"
