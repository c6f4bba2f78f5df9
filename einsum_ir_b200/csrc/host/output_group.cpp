// C-ABI: the output group of a sharded contraction (eir_output_group_*). Every
// rank's full output buffer is mapped into every process with CUDA IPC; the
// handles travel through the caller's all-gather, so any inter-process
// transport can carry them. eir_contract_gather then writes a rank's block
// into the others' buffers with the copy engines.
#include <cstring>
#include <vector>
#include "eir_cuda.h"
#include "eir_plan.h"

struct eir_output_group {
  int32_t rank = 0, world = 1;
  std::vector<char *> ptrs;   // per rank: the buffer as seen from this process (own: out)
  std::vector<void *> bases;  // mappings to close
};

namespace {

// what each rank contributes to the exchange
struct HandleRecord {
  int32_t ok = 0;
  int32_t pad = 0;
  int64_t offset = 0;
  unsigned char handle[EIR_IPC_HANDLE_BYTES] = {};
};

void close_all(eir_output_group *g) {
  for (void *b : g->bases) eir_ipc_close_handle(b);
  g->bases.clear();
}

}  // namespace

extern "C" {

int eir_output_group_create(int32_t rank, int32_t world, void *out, eir_allgather_fn allgather, void *user,
                            eir_output_group **group) {
  if (group == nullptr || out == nullptr || world < 1 || rank < 0 || rank >= world ||
      (world > 1 && allgather == nullptr))
    return eir::api_set_error(EIR_INVALID_ARGUMENT, "eir_output_group_create: bad argument");
  *group = nullptr;
  auto *g = new eir_output_group();
  g->rank = rank;
  g->world = world;
  g->ptrs.assign((size_t)world, nullptr);
  g->ptrs[(size_t)rank] = static_cast<char *>(out);
  if (world > 1) {
    HandleRecord mine;
    mine.ok = eir_ipc_get_handle(out, mine.handle, &mine.offset) == EIR_SUCCESS ? 1 : 0;
    std::vector<HandleRecord> all((size_t)world);
    if (allgather(&mine, all.data(), (int64_t)sizeof(HandleRecord), user) != 0) {
      delete g;
      return eir::api_set_error(EIR_UNDEFINED_ERROR, "eir_output_group_create: the all-gather failed");
    }
    int32_t ok = 1;
    for (auto const &r : all) ok &= r.ok;
    for (int32_t r = 0; r < world && ok; ++r) {
      if (r == rank) continue;
      void *ptr = nullptr, *base = nullptr;
      if (eir_ipc_open_handle(all[(size_t)r].handle, all[(size_t)r].offset, &ptr, &base) != EIR_SUCCESS) {
        ok = 0;
        break;
      }
      g->ptrs[(size_t)r] = static_cast<char *>(ptr);
      g->bases.push_back(base);
    }
    // every rank learns whether every rank mapped every buffer
    std::vector<int32_t> flags((size_t)world, 0);
    if (allgather(&ok, flags.data(), (int64_t)sizeof(int32_t), user) != 0) {
      close_all(g);
      delete g;
      return eir::api_set_error(EIR_UNDEFINED_ERROR, "eir_output_group_create: the all-gather failed");
    }
    for (int32_t f : flags) ok &= f;
    if (!ok) {
      close_all(g);
      delete g;
      return eir::api_set_error(EIR_CUDA_ERROR, "eir_output_group_create: a rank could not export or map "
                                                "the output buffers (CUDA IPC)");
    }
  }
  *group = g;
  return EIR_SUCCESS;
}

int eir_output_group_peers(eir_output_group const *g, int64_t offset, void **peers) {
  if (g == nullptr || offset < 0 || (g->world > 1 && peers == nullptr))
    return eir::api_set_error(EIR_INVALID_ARGUMENT, "eir_output_group_peers: bad argument");
  int32_t k = 0;
  for (int32_t r = 0; r < g->world; ++r)
    if (r != g->rank) peers[k++] = g->ptrs[(size_t)r] + offset;
  return EIR_SUCCESS;
}

int eir_output_group_destroy(eir_output_group *g) {
  if (g == nullptr) return EIR_SUCCESS;
  close_all(g);
  delete g;
  return EIR_SUCCESS;
}

}  // extern "C"
