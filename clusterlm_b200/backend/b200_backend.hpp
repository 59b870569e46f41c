#pragma once
// B200 backend: the `--backend b200` BackendAdapter of ClusterLM over libclm_b200.so.
//
// Implements the reference's BackendAdapter / ExecutionDomain interfaces
// (runtime/domain/include/clusterlm/domain/backend_adapter.hpp:14-27, execution_domain.hpp:143-174) with
// the device engines of libclm_b200 behind the C ABI (include/clm_b200.h).  Admission (epochs, window IDs,
// state versions, idempotent commits) is delegated to windows::WindowLedger exactly as the reference
// domain does (runtime/domain/src/reference_domain.cpp:379), so the transaction rules are identical.
//
// This translation unit is compiled against the reference's headers and links its runtime (ledger, status,
// boundary codec); it is the code a maintainer adds as runtime/backends/b200 (see the integration notes).
#include <filesystem>
#include <memory>
#include <vector>

#include "clusterlm/domain/backend_adapter.hpp"
#include "clusterlm/domain/drafter.hpp"

namespace clusterlm::backends {

struct B200BackendOptions {
  // CUDA device of each domain, by StageId (stage index); stages beyond the list use `default_device`.
  std::vector<int> stage_devices;
  int default_device = 0;
  // Directory of the GGUF files a llama.cpp manifest names (ModelManifest::shards), as LlamaBackendOptions'
  // model_dir (runtime/backends/llama/src/llama_backend.cpp:307).  Read for the tensor directory and metadata
  // only: the tensor bytes come from the domain's ObjectResolver at prepare.  Unused for the fixture family.
  std::filesystem::path model_dir;
};

// Build hash shared by Father and Nodes (PreparePlan admission).
inline constexpr const char* kB200BuildHash = "b200-sm100a-v1";

std::unique_ptr<domain::BackendAdapter> make_b200_backend(const B200BackendOptions& options = {});

// GPU MTP drafter bound to a prepared b200 tail domain (the "b200" case of make_backend_drafter,
// backend_factory.hpp:49): greedy chained draft steps of MtpFixtureDrafter (drafter.cpp:39-89) on the tail's GPU.
// kFailedPrecondition when mtp_drafter / token_embd were not provisioned to the tail.  The tail must outlive it.
Result<std::unique_ptr<domain::Drafter>> make_b200_mtp_drafter(domain::ExecutionDomain& tail);
// The same drafter standalone, from the model store, on `device` (at most `max_draft` steps per device call).
Result<std::unique_ptr<domain::Drafter>> make_b200_mtp_drafter(const objects::ModelManifest& manifest,
                                                               const objects::ObjectResolver& resolver, int device = 0,
                                                               std::uint32_t max_draft = 16);

}  // namespace clusterlm::backends
