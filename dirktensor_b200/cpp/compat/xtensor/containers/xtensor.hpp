// Minimal stand-in for xtensor's xt::xtensor<T, N>, used only to build and test
// the drop-in classes in this repository (xtensor is not installed here).  A
// project that uses the drop-in compiles it against the real xtensor instead;
// the drop-in code relies only on API that both provide: shape(i), shape(),
// size(), data(), operator(), and xt::empty / xt::zeros with a braced shape.
// The element-wise sum of two tensors of one shape is here too, because the
// reference's OlmoBlock (which holds the drop-in OlmoAttention) adds residuals.
#pragma once

#include <array>
#include <cstddef>
#include <vector>

namespace xt {

template <class T, std::size_t N>
class xtensor {
public:
    using value_type = T;
    using shape_type = std::array<std::size_t, N>;

    xtensor() { dims_.fill(0); }
    explicit xtensor(const shape_type& s) : dims_(s) {
        std::size_t n = 1;
        for (std::size_t d : dims_) n *= d;
        buf_.resize(n);
    }

    std::size_t shape(std::size_t i) const { return dims_[i]; }
    const shape_type& shape() const { return dims_; }
    std::size_t size() const { return buf_.size(); }
    std::size_t dimension() const { return N; }
    T* data() { return buf_.data(); }
    const T* data() const { return buf_.data(); }

    template <class... I>
    T& operator()(I... i) { return buf_[flat(i...)]; }
    template <class... I>
    const T& operator()(I... i) const { return buf_[flat(i...)]; }

private:
    template <class... I>
    std::size_t flat(I... i) const {
        static_assert(sizeof...(I) == N, "rank mismatch");
        const std::size_t idx[N] = {static_cast<std::size_t>(i)...};
        std::size_t o = 0;
        for (std::size_t k = 0; k < N; ++k) o = o * dims_[k] + idx[k];
        return o;
    }
    shape_type dims_;
    std::vector<T> buf_;
};

template <class T, std::size_t N>
xtensor<T, N> operator+(const xtensor<T, N>& a, const xtensor<T, N>& b) {
    xtensor<T, N> r(a.shape());
    for (std::size_t i = 0; i < r.size(); ++i) r.data()[i] = a.data()[i] + b.data()[i];
    return r;
}

template <class T, std::size_t L>
xtensor<T, L> empty(const std::size_t (&shape)[L]) {
    std::array<std::size_t, L> s{};
    for (std::size_t i = 0; i < L; ++i) s[i] = shape[i];
    return xtensor<T, L>(s);
}

template <class T, std::size_t L>
xtensor<T, L> zeros(const std::size_t (&shape)[L]) {
    return empty<T, L>(shape);  // std::vector value-initialises: all zeros
}

}  // namespace xt
