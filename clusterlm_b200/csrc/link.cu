// link.cu — stage-to-stage message links over NVLink peer memory (link.cuh), and their C ABI.
#include <unistd.h>

#include <cstring>

#include "link.cuh"
#include "pdl.cuh"

struct clm_b200_link {
  clm_b200_ctx* ctx = nullptr;
  int end = CLM_LINK_SEND;
  uint32_t nslots = 0;
  uint32_t slot_bytes = 0;
  unsigned long long timeout_ns = 0;
  uint8_t* own = nullptr;   // receiver: flags + slots; sender: credit word (cudaMalloc, exported)
  size_t own_bytes = 0;
  uint8_t* local = nullptr;  // this end's sequence counter (8 B) + CTA arrivals (8 B)
  uint8_t* peer = nullptr;   // the other end's exported allocation, mapped here
  bool peer_ipc = false;     // peer mapped by cudaIpcOpenMemHandle (else a same-process pointer)
};

namespace clm {

namespace {

constexpr uint32_t kLinkMagic = 0x4b4e494c;  // "LINK"

// Bytes of the receiver's flag array (kept a multiple of 256 so the slots stay 16-byte aligned).
size_t flags_bytes(uint32_t nslots) { return ((size_t)nslots * 8 + 255) / 256 * 256; }

struct LinkHandle {  // CLM_B200_LINK_HANDLE_BYTES, exported by one end and read by the other
  uint32_t magic;
  int32_t end;
  int32_t device;
  int32_t pid;
  uint32_t nslots;
  uint32_t slot_bytes;
  uint64_t ptr;  // the exported allocation in the exporting process
  uint8_t uuid[16];
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(LinkHandle) <= CLM_B200_LINK_HANDLE_BYTES, "link handle too large");

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const uint64_t* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Polls *p >= target; false (and *err = kErrLinkTimeout) after the deadline or the iteration cap, or at once when
// an earlier wait has already failed.
__device__ bool link_wait(const uint64_t* p, unsigned long long target, unsigned long long timeout_ns, int* err) {
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0; i < (1u << 27); ++i) {
    if (ld_acquire_sys(p) >= target) return true;
    if (*(volatile int*)err != 0) return false;
    if (global_ns() - t0 > timeout_ns) break;
    __nanosleep(128);
  }
  atomicCAS(err, 0, kErrLinkTimeout);
  return false;
}

// Copies `bytes` (a multiple of 16) with the launch's kLinkCtas x kLinkThreads threads, 16 bytes per access.
__device__ __forceinline__ void link_copy(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, uint32_t bytes) {
  const uint32_t n = bytes / 16;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) d[i] = __ldcg(s + i);
}

__global__ void __launch_bounds__(kLinkThreads) link_send_kernel(LinkDev L, const uint8_t* __restrict__ src,
                                                                 uint32_t bytes, const uint32_t* __restrict__ d_commit,
                                                                 uint32_t q, uint32_t kind, int* err) {
  griddep_wait();
  griddep_launch();  // the next kernel may stage its weights while this one waits; it still waits for our end
  __shared__ bool s_ok;
  const unsigned long long seq = *L.seq + 1;
  const uint32_t slot = (uint32_t)((seq - 1) % L.nslots);
  uint8_t* dst = L.slots + (size_t)slot * L.slot_bytes;
  if (threadIdx.x == 0) {
    // credit: message seq reuses the slot of message seq - nslots, which the receiver must have consumed
    s_ok = seq <= L.nslots || link_wait(L.credit, seq - L.nslots, L.timeout_ns, err);
  }
  __syncthreads();
  if (s_ok) {
    link_copy(dst + kLinkHeaderBytes, src, bytes);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      LinkHeader h{bytes, d_commit ? *d_commit : 0u, q, kind};
      *reinterpret_cast<LinkHeader*>(dst) = h;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(L.arrive, 1u);
    if (prev + 1 == (unsigned)(kLinkCtas * seq)) {
      // every CTA's stores are ordered before this release of the slot's sequence number
      __threadfence_system();
      if (s_ok) st_release_sys(L.flags + slot, seq);
      *L.seq = seq;
    }
  }
}

__global__ void __launch_bounds__(kLinkThreads) link_recv_kernel(LinkDev L, uint8_t* __restrict__ dst,
                                                                 uint32_t max_bytes, uint32_t q, long long* pos,
                                                                 uint32_t* commit_out, int* err) {
  griddep_wait();
  griddep_launch();
  __shared__ bool s_ok;
  const unsigned long long seq = *L.seq + 1;
  const uint32_t slot = (uint32_t)((seq - 1) % L.nslots);
  const uint8_t* src = L.slots + (size_t)slot * L.slot_bytes;
  if (threadIdx.x == 0) s_ok = link_wait(L.flags + slot, seq, L.timeout_ns, err);
  __syncthreads();
  LinkHeader h{0, 0, 0, 0};
  if (s_ok) {
    const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(src));
    h = LinkHeader{raw.x, raw.y, raw.z, raw.w};
    if (h.q != q || h.bytes > max_bytes) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(err, 0, kErrLinkMismatch);
    } else {
      link_copy(dst, src + kLinkHeaderBytes, h.bytes);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(L.arrive, 1u);
    if (prev + 1 == (unsigned)(kLinkCtas * seq)) {
      __threadfence();
      if (s_ok && h.q == q) {
        if (pos) *pos += h.commit;
        if (commit_out) *commit_out = h.commit;
      }
      st_release_sys(L.credit, seq);  // the slot may be reused
      *L.seq = seq;
    }
  }
}

}  // namespace

int link_dev(const clm_b200_link* link, bool sender, LinkDev* out) {
  CLM_CHECK(link != nullptr && out != nullptr, CLM_INVALID_ARGUMENT, "null link");
  CLM_CHECK(link->peer != nullptr, CLM_FAILED_PRECONDITION, "link is not connected");
  CLM_CHECK((link->end == CLM_LINK_SEND) == sender, CLM_INVALID_ARGUMENT,
            sender ? "a receiving link was given where a sending one is needed"
                   : "a sending link was given where a receiving one is needed");
  LinkDev L;
  uint8_t* rx = sender ? link->peer : link->own;
  uint8_t* tx = sender ? link->own : link->peer;
  L.flags = reinterpret_cast<uint64_t*>(rx);
  L.slots = rx + flags_bytes(link->nslots);
  L.credit = reinterpret_cast<uint64_t*>(tx);
  L.seq = reinterpret_cast<unsigned long long*>(link->local);
  L.arrive = reinterpret_cast<unsigned*>(link->local + 8);
  L.nslots = link->nslots;
  L.slot_bytes = link->slot_bytes;
  L.timeout_ns = link->timeout_ns;
  *out = L;
  return CLM_OK;
}

int launch_link_send(const LinkDev& L, const void* src, uint32_t bytes, const uint32_t* d_commit, uint32_t q,
                     uint32_t kind, int* err, cudaStream_t st) {
  CLM_CHECK(bytes % 16 == 0 && bytes + kLinkHeaderBytes <= L.slot_bytes, CLM_RESOURCE_EXHAUSTED,
            "message larger than the link's slot");
  return launch_pdl(link_send_kernel, dim3(kLinkCtas), dim3(kLinkThreads), 0, st, L,
                    static_cast<const uint8_t*>(src), bytes, d_commit, q, kind, err);
}

int launch_link_recv(const LinkDev& L, void* dst, uint32_t max_bytes, uint32_t q, long long* pos,
                     uint32_t* commit_out, int* err, cudaStream_t st) {
  return launch_pdl(link_recv_kernel, dim3(kLinkCtas), dim3(kLinkThreads), 0, st, L, static_cast<uint8_t*>(dst),
                    max_bytes, q, pos, commit_out, err);
}

}  // namespace clm

using namespace clm;

extern "C" {

int clm_b200_link_create(clm_b200_ctx* ctx, int end, uint32_t slots, uint64_t payload_bytes, double timeout_s,
                         clm_b200_link** out) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(out != nullptr, CLM_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  CLM_CHECK(end == CLM_LINK_SEND || end == CLM_LINK_RECV, CLM_INVALID_ARGUMENT, "unknown link end");
  CLM_CHECK(slots >= 1 && slots <= 1024, CLM_INVALID_ARGUMENT, "slots must be in [1, 1024]");
  CLM_CHECK(payload_bytes >= 16 && payload_bytes <= (1ull << 30), CLM_INVALID_ARGUMENT,
            "payload must be in [16 B, 1 GiB]");
  CLM_CHECK(timeout_s > 0.0 && timeout_s <= 600.0, CLM_INVALID_ARGUMENT, "timeout must be in (0, 600] seconds");
  auto* l = new clm_b200_link();
  l->ctx = ctx;
  l->end = end;
  l->nslots = slots;
  l->slot_bytes = (uint32_t)(((payload_bytes + 15) / 16) * 16 + kLinkHeaderBytes);
  l->timeout_ns = (unsigned long long)(timeout_s * 1e9);
  l->own_bytes = end == CLM_LINK_RECV ? flags_bytes(slots) + (size_t)slots * l->slot_bytes : 256;
  cudaError_t e = cudaMalloc(&l->own, l->own_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&l->local, 16);
  if (e == cudaSuccess) e = cudaMemset(l->own, 0, l->own_bytes);
  if (e == cudaSuccess) e = cudaMemset(l->local, 0, 16);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (l->own) cudaFree(l->own);
    if (l->local) cudaFree(l->local);
    delete l;
    return cuda_fail(e, "link allocation");
  }
  ctx_retain(ctx);
  *out = l;
  return CLM_OK;
}

int clm_b200_link_export(const clm_b200_link* link, void* handle) {
  CLM_CHECK(link != nullptr && handle != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  CLM_TRY(ctx_enter(link->ctx));
  LinkHandle h;
  std::memset(&h, 0, sizeof(h));
  h.magic = kLinkMagic;
  h.end = link->end;
  h.device = link->ctx->device;
  h.pid = (int32_t)getpid();
  h.nslots = link->nslots;
  h.slot_bytes = link->slot_bytes;
  h.ptr = reinterpret_cast<uint64_t>(link->own);
  cudaDeviceProp prop;
  CLM_CUDA(cudaGetDeviceProperties(&prop, link->ctx->device));
  std::memcpy(h.uuid, &prop.uuid, sizeof(h.uuid));
  CLM_CUDA(cudaIpcGetMemHandle(&h.ipc, link->own));
  std::memset(handle, 0, CLM_B200_LINK_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  return CLM_OK;
}

int clm_b200_link_connect(clm_b200_link* link, const void* peer_handle) {
  CLM_CHECK(link != nullptr && peer_handle != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  CLM_TRY(ctx_enter(link->ctx));
  CLM_CHECK(link->peer == nullptr, CLM_FAILED_PRECONDITION, "link already connected");
  LinkHandle h;
  std::memcpy(&h, peer_handle, sizeof(h));
  CLM_CHECK(h.magic == kLinkMagic, CLM_INVALID_ARGUMENT, "not a link handle");
  CLM_CHECK(h.end != link->end, CLM_INVALID_ARGUMENT, "both ends of the link have the same direction");
  CLM_CHECK(h.nslots == link->nslots && h.slot_bytes == link->slot_bytes, CLM_VERSION_MISMATCH,
            "link ends disagree on slots or slot size");
  cudaDeviceProp prop;
  CLM_CUDA(cudaGetDeviceProperties(&prop, link->ctx->device));
  // The receiver's wait spins until the sender's kernel runs; both on one GPU, nothing guarantees they run
  // concurrently, so a link always joins two different GPUs.
  CLM_CHECK(std::memcmp(h.uuid, &prop.uuid, sizeof(h.uuid)) != 0, CLM_INVALID_ARGUMENT,
            "both ends of the link are on the same GPU");
  if (h.pid == (int32_t)getpid()) {
    int can = 0;
    CLM_CUDA(cudaDeviceCanAccessPeer(&can, link->ctx->device, h.device));
    CLM_CHECK(can, CLM_HARDWARE_UNAVAILABLE, "no peer access between the link's GPUs");
    cudaError_t e = cudaDeviceEnablePeerAccess(h.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      return cuda_fail(e, "cudaDeviceEnablePeerAccess");
    }
    link->peer = reinterpret_cast<uint8_t*>(h.ptr);
    link->peer_ipc = false;
  } else {
    void* p = nullptr;
    CLM_CUDA(cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess));
    link->peer = static_cast<uint8_t*>(p);
    link->peer_ipc = true;
  }
  return CLM_OK;
}

int clm_b200_link_destroy(clm_b200_link* link) {
  if (link == nullptr) return CLM_OK;
  cudaSetDevice(link->ctx->device);
  cudaDeviceSynchronize();
  if (link->peer && link->peer_ipc) cudaIpcCloseMemHandle(link->peer);
  if (link->own) cudaFree(link->own);
  if (link->local) cudaFree(link->local);
  clm_b200_ctx* ctx = link->ctx;
  delete link;
  ctx_release(ctx);
  return CLM_OK;
}

}  // extern "C"
