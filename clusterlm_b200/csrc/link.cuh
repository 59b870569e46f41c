// link.cuh — stage-to-stage message links between GPUs of one node (link.cu).
//
// A link is a one-way FIFO of `slots` messages from a sender GPU to a receiver GPU.  It replaces the
// RunWindow / StageResult TCP hop of the reference (orchestrator/coordinator/src/coordinator.cpp:736-832,
// runtime/transport) for stages placed on GPUs of one box: the sender's kernel stores the message straight into
// the receiver's memory over NVLink (peer stores, no multicast, no TMA), then publishes the slot's sequence
// number with a system-scope release; the receiver's kernel polls that flag in its own memory, copies the
// message out and returns a credit (the consumed sequence number) into the sender's memory.
//
// Memory: the receiver owns [flags: slots x u64][slot 0][slot 1]... (each slot = 16-byte header + payload); the
// sender owns the credit word.  Each end also keeps a local sequence counter and a CTA-arrival counter.
// Every wait is bounded (iterations and %globaltimer nanoseconds) and reports through the caller's error flag.
#pragma once
#include "common.cuh"

struct clm_b200_link;

namespace clm {

constexpr int kErrLinkTimeout = 4;   // error-flag value: a link wait (message or credit) gave up
constexpr int kErrLinkMismatch = 5;  // error-flag value: a message's window width differs from the receiver's
constexpr int kLinkCtas = 16;        // CTAs of every link kernel (fixed: arrivals count to kLinkCtas * seq)
constexpr int kLinkThreads = 256;
constexpr uint32_t kLinkHeaderBytes = 16;

enum { LINK_MSG_WINDOW = 0, LINK_MSG_PREFILL = 1 };

struct LinkHeader {
  uint32_t bytes;   // payload bytes
  uint32_t commit;  // positions the receiver commits for the session before running this window
  uint32_t q;       // window width
  uint32_t kind;    // LINK_MSG_*
};

// The device view of one end.
struct LinkDev {
  uint64_t* flags = nullptr;          // receiver's flags (sender: mapped peer memory)
  uint8_t* slots = nullptr;           // receiver's slots (sender: mapped peer memory)
  uint64_t* credit = nullptr;         // sender's credit word (receiver: mapped peer memory)
  unsigned long long* seq = nullptr;  // this end's last sequence number (local)
  unsigned* arrive = nullptr;         // this end's CTA arrivals (local, monotonic)
  uint32_t nslots = 0;
  uint32_t slot_bytes = 0;            // header + payload capacity
  unsigned long long timeout_ns = 0;
};

// The device view of `link` (the link must be connected).
int link_dev(const clm_b200_link* link, bool sender, LinkDev* out);

// Sends `bytes` from `src` (device) as the next message: header {bytes, commit (*d_commit, or 0 when null), q, kind}.
int launch_link_send(const LinkDev& L, const void* src, uint32_t bytes, const uint32_t* d_commit, uint32_t q,
                     uint32_t kind, int* err, cudaStream_t st);
// Receives the next message into `dst` (at most `max_bytes`); checks its window width against `q`.  With
// `pos` non-null the message's commit count is added to *pos (the session's committed position) before the
// kernel ends; `commit_out` (optional) receives the count.
int launch_link_recv(const LinkDev& L, void* dst, uint32_t max_bytes, uint32_t q, long long* pos,
                     uint32_t* commit_out, int* err, cudaStream_t st);

}  // namespace clm
