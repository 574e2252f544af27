// TEST INFRASTRUCTURE (oracle) -- not part of the product.
// Minimal stand-in for oneTBB's tbb::blocked_range, written for this
// repository so the reference's FlashAttention.cpp compiles in place.
#pragma once
#include <cstddef>

namespace tbb {

template <class Value>
class blocked_range {
public:
    blocked_range(Value begin, Value end, std::size_t grainsize = 1)
        : begin_(begin), end_(end), grain_(grainsize ? grainsize : 1) {}
    Value begin() const { return begin_; }
    Value end() const { return end_; }
    std::size_t size() const { return static_cast<std::size_t>(end_ - begin_); }
    bool empty() const { return !(begin_ < end_); }
    std::size_t grainsize() const { return grain_; }

private:
    Value begin_, end_;
    std::size_t grain_;
};

}  // namespace tbb
