// Compile-only stand-in for the reference's Metal pipeline executor.  The host
// generators never dispatch through it; the pipeline lookup the file also
// defines returns null here and is never called by the oracle shim.
#pragma once
#include <string_view>

#include <Metal/Metal.h>

namespace muda::libraries {
class LibraryExecutor {
 public:
  static LibraryExecutor& Instance() noexcept {
    static LibraryExecutor executor;
    return executor;
  }
  id<MTLComputePipelineState> GetOrLoadPipeline(std::string_view, std::string_view,
                                                std::string_view) noexcept {
    return nullptr;
  }
};
}  // namespace muda::libraries
