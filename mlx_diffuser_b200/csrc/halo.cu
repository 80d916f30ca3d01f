// Halo exchange of a Morton-partitioned scene over NVLink peer memory.
//
// A rank's halo rows (rows owned by other ranks that are kernel neighbours of its own rows)
// must be refreshed before every convolution. Here the owner pushes them: one kernel gathers
// the rows a peer needs from the owner's local buffer and stores them straight into the peer's
// halo block through a CUDA IPC mapping of the peer's buffer (P2P stores over NVLink), and a
// second kernel raises the peer's "data" flag with a system-scope release. The receiver's
// boundary rows wait on that flag (acquire, bounded) and, once they are convolved, the receiver
// raises an "ack" flag in the owner, which the owner waits for before its next push into the same
// buffer. Flags hold the exchange's epoch, so nothing is ever reset.
//
// Order on each rank's stream for one exchange of epoch e:
//   wait ack[p] >= e-1 (peers finished with my previous push) -> push rows -> data[me]@p := e
//   -> interior convolution -> wait data[p] >= e (peers' rows arrived) -> boundary convolution
//   -> ack[me]@p := e.
// No rank waits for work that is queued behind its own wait, so the exchange cannot deadlock;
// every wait is bounded (2 s) and reports SV_DEVICE_WAIT_TIMEOUT instead of hanging. Only this
// library's own kernels touch peer memory, with plain stores; there is no multicast.
#include <cstring>

#include "common.cuh"

namespace sv {
namespace {

constexpr int MAX_PEERS = 8;

struct PeerBases {
  uint8_t* base[MAX_PEERS];
  int64_t rows[MAX_PEERS];  // rows of each peer buffer: stores beyond it are refused
};

struct FlagPtrs {
  int64_t* ptr[MAX_PEERS];
};

// Row j of the send list: local row rows[j] goes to row dst_rows[j] of peer peers[j]'s buffer.
template <int BYTES>
__global__ void halo_push_kernel(const uint8_t* __restrict__ local, int row_bytes,
                                 const int32_t* __restrict__ rows,
                                 const int32_t* __restrict__ dst_rows,
                                 const int32_t* __restrict__ peers, int64_t m, int npeers,
                                 int64_t local_rows, PeerBases pb, int32_t* status) {
  const int chunks = row_bytes / BYTES;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < m * chunks) {
    const int64_t j = t / chunks;
    const int c = (int)(t - j * chunks);
    const int32_t r = __ldg(&rows[j]);
    const int32_t p = __ldg(&peers[j]);
    const int32_t d = __ldg(&dst_rows[j]);
    if (r < 0 || r >= local_rows || p < 0 || p >= npeers || d < 0 || d >= pb.rows[p]) {
      report(status, SV_DEVICE_BAD_INDEX);  // nothing is written outside a peer's buffer
    } else {
      const uint8_t* src = local + (int64_t)r * row_bytes + (int64_t)c * BYTES;
      uint8_t* dst = pb.base[p] + (int64_t)d * row_bytes + (int64_t)c * BYTES;
      if constexpr (BYTES == 16)
        *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
      else
        *dst = *src;
      __threadfence_system();  // the peer store is visible before the flag kernel runs
    }
  }
}

__global__ void halo_signal_kernel(FlagPtrs flags, int count, int64_t value) {
  const int i = threadIdx.x;
  if (i < count) {
    __threadfence_system();
    asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(flags.ptr[i]), "l"(value)
                 : "memory");
  }
}

__global__ void halo_wait_kernel(FlagPtrs flags, int count, int64_t value, int32_t* status) {
  const int i = threadIdx.x;
  if (i >= count) return;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    int64_t v;
    asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(flags.ptr[i]) : "memory");
    if (v >= value) return;
    if (global_timer_ns() - t0 > 2000000000ull) {
      report(status, SV_DEVICE_WAIT_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

typedef int (*GetAddressRangeFn)(unsigned long long*, size_t*, unsigned long long);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  }
  return fn;
}

}  // namespace
}  // namespace sv

using namespace sv;

extern "C" int sv_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_ipc_handle: null pointer");
  GetAddressRangeFn range = address_range_fn();
  if (!range) SV_FAIL(SV_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, (unsigned long long)(uintptr_t)ptr) != 0)
    SV_FAIL(SV_ERR_CUDA, "sv_ipc_handle: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  SV_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)((uintptr_t)ptr - (uintptr_t)base);
  return SV_OK;
}

extern "C" int sv_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  SV_CUDA_TRY(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return SV_OK;
}

extern "C" int sv_ipc_close(void* base) {
  if (!base) return SV_OK;
  SV_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return SV_OK;
}

extern "C" int sv_halo_push(const void* local, int64_t local_rows, int row_bytes,
                            const int32_t* rows, const int32_t* dst_rows, const int32_t* peers,
                            int64_t m, void* const* peer_bases, const int64_t* peer_rows,
                            int npeers, int32_t* status, sv_stream_t stream) {
  if (m < 0 || row_bytes <= 0 || npeers < 0 || npeers > MAX_PEERS || local_rows < 0)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_push: bad sizes");
  if (m == 0) return SV_OK;
  if (!local || !rows || !dst_rows || !peers || !peer_bases || !peer_rows)
    SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_push: null pointer");
  PeerBases pb{};
  bool aligned = aligned16(local) && row_bytes % 16 == 0;
  for (int i = 0; i < npeers; ++i) {
    pb.base[i] = static_cast<uint8_t*>(peer_bases[i]);
    pb.rows[i] = pb.base[i] ? peer_rows[i] : 0;
    aligned = aligned && (pb.base[i] == nullptr || aligned16(pb.base[i]));
  }
  cudaStream_t s = to_stream(stream);
  const int64_t threads = m * (aligned ? row_bytes / 16 : row_bytes);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (aligned)
    halo_push_kernel<16><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(local), row_bytes,
                                                rows, dst_rows, peers, m, npeers, local_rows, pb,
                                                status);
  else
    halo_push_kernel<1><<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(local), row_bytes,
                                               rows, dst_rows, peers, m, npeers, local_rows, pb,
                                               status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int sv_halo_signal(int64_t* const* flags, int count, int64_t value,
                              sv_stream_t stream) {
  if (count < 0 || count > MAX_PEERS) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_signal: count");
  if (count == 0) return SV_OK;
  FlagPtrs f{};
  for (int i = 0; i < count; ++i) {
    if (!flags[i]) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_signal: null flag");
    f.ptr[i] = flags[i];
  }
  halo_signal_kernel<<<1, 32, 0, to_stream(stream)>>>(f, count, value);
  SV_LAUNCH_CHECK();
  return SV_OK;
}

extern "C" int sv_halo_wait(int64_t* const* flags, int count, int64_t value, int32_t* status,
                            sv_stream_t stream) {
  if (count < 0 || count > MAX_PEERS) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_wait: count");
  if (count == 0) return SV_OK;
  FlagPtrs f{};
  for (int i = 0; i < count; ++i) {
    if (!flags[i]) SV_FAIL(SV_ERR_INVALID_ARGUMENT, "sv_halo_wait: null flag");
    f.ptr[i] = flags[i];
  }
  halo_wait_kernel<<<1, 32, 0, to_stream(stream)>>>(f, count, value, status);
  SV_LAUNCH_CHECK();
  return SV_OK;
}
