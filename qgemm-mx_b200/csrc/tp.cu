// tp.cu -- tensor-parallel W4A16 GEMM over the GPUs of one node, W sharded
// along N, with the all-gather of Y done over NVLink peer memory.
//
// Rank r holds rows [r N/world, (r+1) N/world) of W.  The TMA decode and
// stream-K tcgen05 kernels store their bf16 results straight into every
// rank's Y_full [M][N] at columns [r N/world, (r+1) N/world) through the peer
// mappings (NVLink P2P stores) and finish with the arrival exchange of
// tp.cuh.  The other kernels write the slice into a staging buffer in the
// workspace, and k_tp_gather copies it to every rank and does the same
// exchange.  No library collective, no TMA on peer memory.
//
// The counts live in device memory, so the launches can be captured in a
// CUDA graph and replayed.  The wait is bounded (~2 s); on timeout the kernel
// records it and qgemm_tp_status reports QGEMM_ERR_TIMEOUT.  Every rank must
// make the same sequence of calls.
//
// Sync block of a rank (qgemm_tp_sync_bytes): uint32 [kTpMaxWorld] arrival
// slots (slot s counts what rank s has delivered to this rank), the expected
// count and a reserved word; zero it once before first use.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstring>

#include "common.cuh"
#include "tp.cuh"

namespace qg {

__device__ unsigned g_tp_fault = 0;

// Copy the [M][n_loc] slice into every rank's Y_full (16-byte granules when
// the row pitch allows, else 2-byte elements), then tp_finish.  Used after
// the kernels that do not write their slice to the peers themselves.
__global__ void __launch_bounds__(256) k_tp_gather(const uint16_t* __restrict__ src, int M, int n_loc, TpOut t) {
  const bool vec = (n_loc % 8 == 0) && (t.ldy % 8 == 0) && (t.col0 % 8 == 0);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    const int gpr = n_loc / 8;  // granules per row
    const size_t total = (size_t)M * gpr;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += stride) {
      const int m = (int)(g / gpr), q = (int)(g % gpr);
      const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)m * n_loc + 8 * q);
      const size_t off = (size_t)m * t.ldy + t.col0 + 8 * q;
      for (int d = 0; d < t.world; ++d) *reinterpret_cast<uint4*>(t.y[d] + off) = v;
    }
  } else {
    const size_t total = (size_t)M * n_loc;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
      const int m = (int)(e / n_loc), n = (int)(e % n_loc);
      const uint16_t v = src[e];
      for (int d = 0; d < t.world; ++d) t.y[d][(size_t)m * t.ldy + t.col0 + n] = v;
    }
  }
  tp_finish(t, &g_tp_fault);
}

qgemm_status_t gemm_decode_ex(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32, void* ws,
                              size_t ws_bytes, cudaStream_t s, const TpOut* tp);
size_t gemm_decode_workspace(const qgemm_weights_t* w, int M);
int32_t gemm_launch_count(const qgemm_weights_t* w, int M, int32_t* kernel);
unsigned umma_sk_fault();
unsigned gemv_tma_fault();
unsigned umma_bs_fault();

cudaError_t tp_fault_clear() {
  const unsigned z = 0;
  return cudaMemcpyToSymbol(g_tp_fault, &z, sizeof(z));
}

static size_t pad256_tp(size_t b) { return (b + 255) & ~(size_t)255; }

// Kernels that store their slice into every rank's Y_full themselves
// (TMA-fed decode, stream-K tcgen05, block-scaled tcgen05); the others go
// through k_tp_gather.
static bool fused_tp(const qgemm_weights_t* w, int M) {
  int32_t k = -1;
  return gemm_launch_count(w, M, &k) > 0 && (k == 1 || k == 2 || k == 4);
}

}  // namespace qg

using namespace qg;

extern "C" {

size_t qgemm_tp_sync_bytes(int32_t world) {
  (void)world;
  return (kTpMaxWorld + 2) * sizeof(uint32_t);
}

size_t qgemm_tp_workspace_size(const qgemm_weights_t* w_local, int32_t M) {
  if (!w_local || M < 1) return 0;
  const size_t inner = gemm_decode_workspace(w_local, M);
  return pad256_tp(inner) + (size_t)M * w_local->N * sizeof(uint16_t);
}

qgemm_status_t qgemm_tp_gemm_w4a16(const qgemm_weights_t* w_local, const uint16_t* X, int32_t M, int32_t world,
                                   int32_t rank, uint16_t* const* y_peers, uint32_t* const* sync_peers, void* ws,
                                   size_t ws_bytes, void* stream) {
  if (!w_local || !X || !y_peers || !sync_peers) return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: null pointer");
  if (world < 1 || world > kTpMaxWorld) return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: world must be 1..%d", kTpMaxWorld);
  if (rank < 0 || rank >= world) return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: rank %d outside 0..%d", rank, world - 1);
  if (M < 1) return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: M must be >= 1");
  const size_t n_loc = w_local->N;
  const size_t N = n_loc * (size_t)world;
  if (N > (size_t)INT32_MAX) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "tp_gemm: N too large");
  TpOut t = {};
  t.world = world;
  t.rank = rank;
  t.col0 = (int)(n_loc * rank);
  t.ldy = (int)N;
  for (int d = 0; d < world; ++d) {
    if (!y_peers[d] || !sync_peers[d]) return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: null peer pointer %d", d);
    if ((reinterpret_cast<uintptr_t>(y_peers[d]) & 15u) || (reinterpret_cast<uintptr_t>(sync_peers[d]) & 3u))
      return fail(QGEMM_ERR_INVALID_ARG, "tp_gemm: peer buffers must be 16-byte (Y) and 4-byte (sync) aligned");
    t.y[d] = y_peers[d];
    t.sync[d] = sync_peers[d];
  }
  const size_t need = qgemm_tp_workspace_size(w_local, M);
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 15u) || ws_bytes < need)
    return fail(QGEMM_ERR_WORKSPACE, "tp_gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", need,
                ws_bytes);
  // [GEMM workspace (tickets first) | this rank's Y slice]
  uint8_t* inner = static_cast<uint8_t*>(ws);
  const size_t inner_bytes = gemm_decode_workspace(w_local, M);
  uint16_t* slice = reinterpret_cast<uint16_t*>(inner + pad256_tp(inner_bytes));
  cudaStream_t s = as_stream(stream);
  if (fused_tp(w_local, M))  // the GEMM kernel writes every rank's Y_full and synchronises
    return gemm_decode_ex(w_local, X, M, nullptr, false, inner, inner_bytes, s, &t);
  qgemm_status_t st = gemm_decode_ex(w_local, X, M, slice, false, inner, inner_bytes, s, nullptr);
  if (st != QGEMM_OK) return st;
  DevProps p;
  st = device_props(&p);
  if (st != QGEMM_OK) return st;
  const size_t granules = ((size_t)M * n_loc + 7) / 8;
  unsigned grid = (unsigned)((granules + 255) / 256);
  const unsigned cap = (unsigned)p.sm_count * 4;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  k_tp_gather<<<grid, 256, 0, s>>>(slice, M, (int)n_loc, t);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_tp_status(int32_t* timed_out) {
  unsigned f = 0;
  QG_CUDA_RET(cudaMemcpyFromSymbol(&f, g_tp_fault, sizeof(f)));
  const unsigned g = umma_sk_fault(), h = gemv_tma_fault(), b = umma_bs_fault();  // the fused kernels' own flags
  if (g == 0xFFFFFFFFu || h == 0xFFFFFFFFu || b == 0xFFFFFFFFu)
    return fail(QGEMM_ERR_CUDA, "tp_status: reading a fault flag failed");
  f |= g | h | b;
  if (timed_out) *timed_out = (int32_t)f;
  return f ? fail(QGEMM_ERR_TIMEOUT, "tp_gemm: a peer did not announce its slice within the bounded wait (~2 s)") : QGEMM_OK;
}

// A pointer inside a larger allocation (a caching allocator's block) is
// shared as (handle of the allocation, byte offset of the pointer in it).
qgemm_status_t qgemm_ipc_handle(const void* dev_ptr, uint8_t* handle64, size_t* offset) {
  if (!dev_ptr || !handle64 || !offset) return fail(QGEMM_ERR_INVALID_ARG, "ipc_handle: null pointer");
  using range_fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static range_fn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return fail(QGEMM_ERR_CUDA, "ipc_handle: cuMemGetAddressRange unavailable");
    fn = reinterpret_cast<range_fn>(p);
  }
  CUdeviceptr base = 0;
  size_t bytes = 0;
  if (fn(&base, &bytes, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(QGEMM_ERR_CUDA, "ipc_handle: pointer is not a device allocation");
  cudaIpcMemHandle_t h;
  QG_CUDA_RET(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == 64, "CUDA IPC handle is 64 bytes");
  std::memcpy(handle64, &h, 64);
  *offset = (size_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return QGEMM_OK;
}

// Maps another process's allocation; *dev_ptr = its base (add the offset).
qgemm_status_t qgemm_ipc_open(const uint8_t* handle64, void** dev_ptr) {
  if (!handle64 || !dev_ptr) return fail(QGEMM_ERR_INVALID_ARG, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, 64);
  QG_CUDA_RET(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return QGEMM_OK;
}

qgemm_status_t qgemm_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return fail(QGEMM_ERR_INVALID_ARG, "ipc_close: null pointer");
  QG_CUDA_RET(cudaIpcCloseMemHandle(dev_ptr));
  return QGEMM_OK;
}

}  // extern "C"
