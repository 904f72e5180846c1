// ctx_cache.h -- a small table of per-CUDA-context addresses (plain C++, no CUDA headers).
//
// A __device__ variable has one instance per context that loads the module, so its device address
// belongs to a context, not to a device ordinal: cudaDeviceReset rebuilds the primary context (and
// the module) with the variable at a possibly different address, and a context made with cuCtxCreate
// on the same ordinal holds its own instance.  The table is therefore keyed on the context's unique
// id (cuCtxGetId), which the driver never reuses within a process.  Ids of contexts that are gone
// simply stop being asked for; when the table is full the oldest entry is overwritten.
#ifndef WISP_CTX_CACHE_H
#define WISP_CTX_CACHE_H

#include <stdint.h>

namespace wisp {

template <int kEntries>
struct ContextAddressTable {
  uint64_t id[kEntries] = {};
  void* addr[kEntries] = {};
  bool used[kEntries] = {};
  int next = 0;  // slot the next insert overwrites once every slot is used

  // address recorded for context `ctx_id`, or nullptr
  void* find(uint64_t ctx_id) const {
    for (int i = 0; i < kEntries; ++i)
      if (used[i] && id[i] == ctx_id) return addr[i];
    return nullptr;
  }

  // record (or replace) the address of context `ctx_id`
  void put(uint64_t ctx_id, void* p) {
    for (int i = 0; i < kEntries; ++i)
      if (used[i] && id[i] == ctx_id) {
        addr[i] = p;
        return;
      }
    for (int i = 0; i < kEntries; ++i)
      if (!used[i]) {
        used[i] = true, id[i] = ctx_id, addr[i] = p;
        return;
      }
    id[next] = ctx_id, addr[next] = p;
    next = (next + 1) % kEntries;
  }
};

}  // namespace wisp

#endif  // WISP_CTX_CACHE_H
