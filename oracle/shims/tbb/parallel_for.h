// TEST INFRASTRUCTURE (oracle) -- not part of the product.
// Minimal stand-in for oneTBB's tbb::parallel_for over a blocked_range,
// written for this repository.  Work is handed out dynamically, one grain at a
// time, from an atomic counter to `ref_shim_threads()` std::threads, which is
// close to TBB's work-stealing behaviour for the reference's loop over B*H.
#pragma once
#include <algorithm>
#include <atomic>
#include <cstddef>
#include <thread>
#include <vector>

#include "blocked_range.h"

// Thread count used by the shim; set from the C wrapper (0 = all cores).
int ref_shim_threads();

namespace tbb {

template <class Value, class Body>
void parallel_for(const blocked_range<Value>& range, const Body& body) {
    const std::size_t n = range.size();
    if (n == 0) return;
    const std::size_t grain = range.grainsize();
    const std::size_t chunks = (n + grain - 1) / grain;
    const std::size_t nthreads = std::min<std::size_t>(chunks, static_cast<std::size_t>(ref_shim_threads()));
    std::atomic<std::size_t> next{0};
    auto worker = [&]() {
        for (;;) {
            const std::size_t c = next.fetch_add(1);
            if (c >= chunks) break;
            const Value b = range.begin() + static_cast<Value>(c * grain);
            const Value e = std::min<Value>(range.end(), b + static_cast<Value>(grain));
            body(blocked_range<Value>(b, e, grain));
        }
    };
    if (nthreads <= 1) { worker(); return; }
    std::vector<std::thread> pool;
    pool.reserve(nthreads - 1);
    for (std::size_t t = 1; t < nthreads; ++t) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
}

}  // namespace tbb
