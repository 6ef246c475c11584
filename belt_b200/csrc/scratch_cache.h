// Per-context record of a device array's address, for belt_latent_decode_noalloc (noalloc.cu).
//
// A `__device__` array has one address per CUDA context that loaded the library's device code: the primary context
// of every device, any context a driver-API host made current, and the new primary context after a cudaDeviceReset
// (the module is loaded again there, possibly at another address). So the record is keyed on the context, not on the
// device ordinal, and a caller refreshes it with a new lookup whenever one is allowed (outside stream capture). While
// a stream is capturing, only a record made earlier in the same context is used; there is none after a reset until
// the next call outside capture. Plain C++ (no CUDA headers), so that its rules are checked by a host-only test.
#pragma once

#include <cstddef>

namespace belt {

template <int kSlots>
class ScratchAddressCache {
 public:
  // Records `addr` as the address in context `ctx` (a fresh lookup), replacing an older record of that context.
  // When every slot is taken, the oldest record is dropped. Returns addr.
  void* refresh(const void* ctx, void* addr) {
    for (int i = 0; i < used_; ++i)
      if (slot_[i].ctx == ctx) {
        slot_[i].addr = addr;
        return addr;
      }
    if (used_ < kSlots) {
      slot_[used_++] = Slot{ctx, addr};
      return addr;
    }
    for (int i = 1; i < kSlots; ++i) slot_[i - 1] = slot_[i];
    slot_[kSlots - 1] = Slot{ctx, addr};
    return addr;
  }

  // The address recorded for `ctx`, or nullptr when this context has none (no lookup made in it yet).
  void* find(const void* ctx) const {
    for (int i = 0; i < used_; ++i)
      if (slot_[i].ctx == ctx) return slot_[i].addr;
    return nullptr;
  }

  // Drops the record of `ctx` (for a context that is known to be gone).
  void forget(const void* ctx) {
    int j = 0;
    for (int i = 0; i < used_; ++i)
      if (slot_[i].ctx != ctx) slot_[j++] = slot_[i];
    used_ = j;
  }

  int size() const { return used_; }

 private:
  struct Slot {
    const void* ctx;
    void* addr;
  };
  Slot slot_[kSlots] = {};
  int used_ = 0;
};

}  // namespace belt
