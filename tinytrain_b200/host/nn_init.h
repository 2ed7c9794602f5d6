// Switch for the reference-identical host initialization of Linear and
// Embedding weights (skipped when a model is built for device-side init).
#pragma once

namespace tt {
namespace detail {
struct HostInitScope {
    explicit HostInitScope(bool host_init);
    ~HostInitScope();
    bool prev;
};
}  // namespace detail
}  // namespace tt
