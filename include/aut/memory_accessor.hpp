// aut/memory_accessor.hpp -- 1D reduced-storage read accessor (host + device).
//
// Drop-in for the reference's include/memory_accessor.hpp:25-48: a
// non-owning, pointer-sized view over a contiguous StorageType array whose
// operator[] returns the element converted to ArithmeticType.  This class
// reproduces the reference's interface verbatim (its typedefs, constructor,
// operator[] and data(), with the same static checks), because code written
// against that interface must compile unchanged; it holds no algorithm.  On
// the GPU the decode-fused DOT reads such arrays through 128-bit loads; this
// accessor is the scalar form of the same contract for user code.
#ifndef AUT_MEMORY_ACCESSOR_HPP_
#define AUT_MEMORY_ACCESSOR_HPP_

#include <cstddef>
#include <type_traits>

#if defined(__CUDACC__)
#define AUT_ACC_HD __host__ __device__
#define AUT_ACC_INLINE __forceinline__
#else
#define AUT_ACC_HD
#define AUT_ACC_INLINE inline
#endif

namespace aut {

template <typename ArithmeticType, typename StorageType> class memory_accessor {
public:
  using arithmetic_type = std::remove_cv_t<ArithmeticType>;
  using storage_type = std::remove_cv_t<StorageType>;
  using pointer = const storage_type *;

  static_assert(std::is_arithmetic_v<arithmetic_type>,
                "ArithmeticType must be an arithmetic type");
  static_assert(std::is_arithmetic_v<storage_type>,
                "StorageType must be an arithmetic type");

  constexpr AUT_ACC_HD explicit memory_accessor(pointer data) noexcept
      : data_{data} {}

  AUT_ACC_HD AUT_ACC_INLINE arithmetic_type
  operator[](std::size_t index) const noexcept {
    return static_cast<arithmetic_type>(data_[index]);
  }

  constexpr AUT_ACC_HD pointer data() const noexcept { return data_; }

private:
  pointer data_;
};

static_assert(sizeof(memory_accessor<double, float>) == sizeof(const float *));
static_assert(std::is_trivially_copyable_v<memory_accessor<double, float>>);
static_assert(std::is_standard_layout_v<memory_accessor<double, float>>);

} // namespace aut

#undef AUT_ACC_HD
#undef AUT_ACC_INLINE

#endif
