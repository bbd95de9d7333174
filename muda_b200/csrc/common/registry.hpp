// registry.hpp — validated opaque handles for every library object.
//
// The reference hands out generation- and kind-tagged tokens instead of raw
// pointers so that a stale, foreign or forged handle is rejected with a status
// code rather than dereferenced (runtime/src/handle_table.hpp:38-42, 101-119).
// This registry keeps that contract with its own token layout:
//
//   bits  0..23  slot number + 1   (so the all-zero token is never valid)
//   bits 24..31  object kind
//   bits 32..63  epoch of the slot (bumped on every release, never 0)
//
// Lookups take a shared lock and hand back a shared_ptr, so an object stays
// alive for the duration of a call even if another thread destroys its handle.
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <vector>

namespace mb200 {

enum class ObjKind : std::uint8_t {
  kBlasHandle = 0x11,
  kFftPlan = 0x21,
  kSparseHandle = 0x31,
  kSparseCsr = 0x32,
  kSparseDnVec = 0x33,
  kSparseDnMat = 0x34,
  kRandGenerator = 0x41,
  kDnnHandle = 0x51,
  kDnnTensor = 0x52,
  kDnnFilter = 0x53,
  kDnnConv = 0x54,
  kDnnActivation = 0x55,
  kDnnPooling = 0x56,
};

template <typename T, ObjKind Kind>
class Registry {
 public:
  static constexpr std::uint64_t kSlotMask = (1ull << 24) - 1ull;

  template <typename Handle>
  Handle add(std::shared_ptr<T> obj) {
    std::unique_lock<std::shared_mutex> guard(mu_);
    std::uint32_t slot;
    if (!free_.empty()) {
      slot = free_.back();
      free_.pop_back();
    } else {
      if (cells_.size() >= kSlotMask - 1) return nullptr;
      slot = static_cast<std::uint32_t>(cells_.size());
      cells_.push_back(Cell{});
    }
    cells_[slot].obj = std::move(obj);
    const std::uint64_t token = (static_cast<std::uint64_t>(cells_[slot].epoch) << 32) |
                                (static_cast<std::uint64_t>(Kind) << 24) |
                                (static_cast<std::uint64_t>(slot) + 1ull);
    return reinterpret_cast<Handle>(static_cast<std::uintptr_t>(token));
  }

  template <typename Handle>
  std::shared_ptr<T> get(Handle h) const noexcept {
    std::uint32_t slot, epoch;
    if (!decode(h, &slot, &epoch)) return nullptr;
    std::shared_lock<std::shared_mutex> guard(mu_);
    if (slot >= cells_.size()) return nullptr;
    const Cell& c = cells_[slot];
    if (c.epoch != epoch || !c.obj) return nullptr;
    return c.obj;
  }

  // Releases the handle; returns the object (null if the handle was not live).
  template <typename Handle>
  std::shared_ptr<T> take(Handle h) noexcept {
    std::uint32_t slot, epoch;
    if (!decode(h, &slot, &epoch)) return nullptr;
    std::unique_lock<std::shared_mutex> guard(mu_);
    if (slot >= cells_.size()) return nullptr;
    Cell& c = cells_[slot];
    if (c.epoch != epoch || !c.obj) return nullptr;
    std::shared_ptr<T> out = std::move(c.obj);
    c.obj.reset();
    c.epoch = (c.epoch == 0xFFFFFFFFu) ? 1u : c.epoch + 1u;
    free_.push_back(slot);
    return out;
  }

 private:
  struct Cell {
    std::uint32_t epoch = 1;
    std::shared_ptr<T> obj;
  };

  template <typename Handle>
  static bool decode(Handle h, std::uint32_t* slot, std::uint32_t* epoch) noexcept {
    const auto token = static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(h));
    if (token == 0) return false;
    if (((token >> 24) & 0xFFull) != static_cast<std::uint64_t>(Kind)) return false;
    const std::uint64_t s = token & kSlotMask;
    const std::uint64_t e = token >> 32;
    if (s == 0 || e == 0) return false;
    *slot = static_cast<std::uint32_t>(s - 1);
    *epoch = static_cast<std::uint32_t>(e);
    return true;
  }

  mutable std::shared_mutex mu_;
  std::vector<Cell> cells_;
  std::vector<std::uint32_t> free_;
};

}  // namespace mb200
