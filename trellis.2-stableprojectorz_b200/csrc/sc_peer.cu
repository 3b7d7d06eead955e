// Halo exchange over peer memory for Morton-sharded convs on one node.
//
// Each rank owns a peer buffer (cudaMalloc, shared by CUDA IPC) holding its
// halo rows and a flag word per source rank.  sc_halo_push stores this rank's
// send rows straight into the destination ranks' buffers over NVLink and, once
// every block has finished (the last block is found with an atomic ticket),
// publishes `epoch` in each destination's flag word for this rank with a
// system-scope release.  sc_halo_wait polls this rank's flag words until all
// peers have published the epoch; the wait is bounded (one second, then
// SC_ETIMEOUT in the handle's device error word).  The conv that follows on
// the same stream reads the halo rows; sc_conv3d_halo instead waits inside the
// conv kernel (sc_conv_tc.cu).  A rank never runs more than one
// exchange ahead of a peer (it waits for the peer's rows of the current
// exchange), so alternating two halo regions per step keeps a peer's reads
// and this rank's writes apart.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <cstring>

namespace sc {
namespace {

constexpr int kPushThreads = 256;

__global__ void __launch_bounds__(kPushThreads) k_halo_push(const uint4* __restrict__ feats, int row_vecs,
                                                            const int32_t* __restrict__ src_row,
                                                            const int32_t* __restrict__ dst_peer,
                                                            const int64_t* __restrict__ dst_off, int64_t n_send,
                                                            void* const* peer_bufs, uint32_t* const* peer_flags,
                                                            int world, int rank, uint32_t epoch,
                                                            unsigned int* ticket, int* err) {
  // one 16-byte vector per thread: consecutive threads cover a row, then the next row
  const int64_t total = n_send * row_vecs;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kPushThreads;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(kPushThreads) + threadIdx.x; e < total; e += stride) {
    const int64_t k = e / row_vecs;
    const int c = static_cast<int>(e - k * row_vecs);
    const int peer = dst_peer[k];
    const int64_t off = dst_off[k];
    // a destination outside the other ranks' buffers or not 16-byte aligned
    // is skipped and reported (SC_EINVAL in the handle's error word)
    if (peer < 0 || peer >= world || peer == rank || off < 0 || (off & 15) != 0) {
      record_error(err, SC_EINVAL);
      continue;
    }
    const uint4 val = __ldg(feats + static_cast<int64_t>(src_row[k]) * row_vecs + c);
    reinterpret_cast<uint4*>(static_cast<uint8_t*>(peer_bufs[peer]) + off)[c] = val;
  }
  // The block barrier orders every thread's row stores before thread 0's
  // system-scope fence (fences are cumulative over what the barrier made
  // visible to thread 0), which orders them before the block's ticket.  The
  // ticket is taken with acquire-release semantics, so the last block's
  // thread 0 also acquires every earlier block's released stores; the block
  // barrier then passes them to the threads that publish the epoch to every
  // peer.  One fence per block rather than one per thread: each system-scope
  // fence waits for the stores it orders to be acknowledged.
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    unsigned int prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ticket) : "memory");
    last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < world && threadIdx.x != rank) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    uint32_t* flag = peer_flags[threadIdx.x] + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
  }
  if (last && threadIdx.x == 0) *ticket = 0u;  // ready for the next push (stream-ordered)
}

__global__ void k_halo_wait(const uint32_t* flags, int world, int rank, uint32_t epoch, int* err) {
  const int r = threadIdx.x;
  if (r >= world || r == rank) return;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
    if (static_cast<int32_t>(v - epoch) >= 0) return;
    if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(err, SC_ETIMEOUT);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace

sc_status peer_alloc(Handle* h, size_t bytes, void** ptr, void* ipc_handle_out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_error(h, e, "peer buffer allocation");
  // zero (flag words included) before any peer can open the buffer
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
  cudaIpcMemHandle_t hd;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&hd, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_error(h, e, "peer buffer IPC handle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= SC_IPC_HANDLE_BYTES, "IPC handle size");
  std::memset(ipc_handle_out, 0, SC_IPC_HANDLE_BYTES);
  std::memcpy(ipc_handle_out, &hd, sizeof(hd));
  *ptr = p;
  return SC_OK;
}

sc_status peer_open(Handle* h, const void* ipc_handle, void** peer_ptr) {
  cudaIpcMemHandle_t hd;
  std::memcpy(&hd, ipc_handle, sizeof(hd));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_error(h, e, "open peer buffer");
  *peer_ptr = p;
  return SC_OK;
}

sc_status halo_push(Handle* h, const void* feats, int row_bytes, const int32_t* src_row, const int32_t* dst_peer,
                    const int64_t* dst_off, int64_t n_send, void* const* peer_bufs, uint32_t* const* peer_flags,
                    int world, int rank, uint32_t epoch) {
  if (!h->push_ticket) {
    // zeroed on the stream the pushes run on, so the first push sees zero
    // whatever kind of stream the caller uses
    cudaError_t e = cudaMalloc(&h->push_ticket, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemsetAsync(h->push_ticket, 0, sizeof(unsigned int), h->stream);
    if (e != cudaSuccess) {
      if (h->push_ticket) cudaFree(h->push_ticket);
      h->push_ticket = nullptr;
      return cuda_error(h, e, "push ticket");
    }
  }
  const int64_t want = (n_send * (row_bytes / 16) + kPushThreads - 1) / kPushThreads;
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, 2 * h->num_sms)));
  ++h->launches;
  k_halo_push<<<blocks, kPushThreads, 0, h->stream>>>(static_cast<const uint4*>(feats), row_bytes / 16, src_row,
                                                      dst_peer, dst_off, n_send, peer_bufs, peer_flags, world, rank,
                                                      epoch, static_cast<unsigned int*>(h->push_ticket), h->derr);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "halo push launch");
}

sc_status halo_wait(Handle* h, const uint32_t* flags, int world, int rank, uint32_t epoch) {
  ++h->launches;
  k_halo_wait<<<1, 32, 0, h->stream>>>(flags, world, rank, epoch, h->derr);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "halo wait launch");
}

}  // namespace sc
