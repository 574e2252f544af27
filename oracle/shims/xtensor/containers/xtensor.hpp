// TEST INFRASTRUCTURE (oracle) -- not part of the product.
//
// Minimal stand-in for xtensor 0.27's `xt::xtensor<T, N>` container, written
// for this repository so that the reference's own FlashAttention.cpp can be
// compiled in place (xtensor is not installed and there is no network).
// It provides exactly the subset that FlashAttention.cpp/.h use:
//   - xt::xtensor<T, N> with shape(i), shape(), variadic operator() returning
//     an lvalue, data(), size();
//   - xt::zeros<T>({...}) / xt::empty<T>({...}) assignable to xtensor<T, N>.
// Storage is dense row-major (the xtensor default), which is what the
// reference's pointer arithmetic (&Q(b, t, h, 0) with row stride H*D) relies on.
#pragma once

#include <array>
#include <cstddef>
#include <initializer_list>
#include <stdexcept>
#include <vector>

namespace xt {

template <class T, std::size_t N>
class xtensor {
public:
    using value_type = T;
    using shape_type = std::array<std::size_t, N>;

    xtensor() { shape_.fill(0); strides_.fill(0); }
    explicit xtensor(const shape_type& shape) { resize(shape); }

    void resize(const shape_type& shape) {
        shape_ = shape;
        std::size_t s = 1;
        for (std::size_t i = N; i-- > 0;) { strides_[i] = s; s *= shape_[i]; }
        data_.assign(s, T(0));
    }

    std::size_t shape(std::size_t i) const { return shape_[i]; }
    const shape_type& shape() const { return shape_; }
    std::size_t size() const { return data_.size(); }
    std::size_t dimension() const { return N; }

    T* data() { return data_.data(); }
    const T* data() const { return data_.data(); }

    template <class... I>
    T& operator()(I... idx) { return data_[offset(idx...)]; }
    template <class... I>
    const T& operator()(I... idx) const { return data_[offset(idx...)]; }

    void fill(T v) { for (auto& x : data_) x = v; }

private:
    template <class... I>
    std::size_t offset(I... idx) const {
        static_assert(sizeof...(I) == N, "index count must equal tensor rank");
        const std::size_t ix[N] = {static_cast<std::size_t>(idx)...};
        std::size_t o = 0;
        for (std::size_t i = 0; i < N; ++i) o += ix[i] * strides_[i];
        return o;
    }

    shape_type shape_;
    shape_type strides_;
    std::vector<T> data_;
};

// Deferred "zeros"/"empty" expression: converts to an xtensor of matching rank.
template <class T>
struct filled_shape {
    std::vector<std::size_t> dims;
    template <std::size_t N>
    operator xtensor<T, N>() const {
        if (dims.size() != N) throw std::runtime_error("xt shim: rank mismatch");
        std::array<std::size_t, N> s{};
        for (std::size_t i = 0; i < N; ++i) s[i] = dims[i];
        return xtensor<T, N>(s);
    }
};

template <class T>
filled_shape<T> zeros(std::initializer_list<std::size_t> dims) { return {std::vector<std::size_t>(dims)}; }

template <class T>
filled_shape<T> empty(std::initializer_list<std::size_t> dims) { return {std::vector<std::size_t>(dims)}; }

}  // namespace xt
