// Stand-in for the subset of the XLA FFI C++ API (xla/ffi/api/ffi.h, shipped
// inside jaxlib) that NanoRTS's kernel sources name.  TEST INFRASTRUCTURE.
//
// jaxlib is not installed here, so the reference's .cu files (core/cuda/step.cu,
// core/cuda/legality.cu, observations/cuda/visibility.cu, adapters/cuda/reset.cu,
// bots/cuda/abstraction_act.cu) cannot include the real header; neither can
// this repository's own XLA FFI handlers (nanorts_b200/ffi/nanorts_b200_ffi.cc),
// which the tests build against this file to drive them without jaxlib.  This file declares the types those files
// use -- buffers, errors, ErrorOr, the remaining-argument lists, the handler
// macro -- with the same names and member functions, so the reference sources
// compile unchanged.  XLA_FFI_DEFINE_HANDLER_SYMBOL does not register an XLA
// handler: it exports the address of the implementation function, which
// oracle/ref_kernels.cu calls directly with buffers it describes itself.
// Nothing here is XLA code; only the interface names are kept.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace xla::ffi {

// Element types named by the reference sources (numbering is this file's own).
enum class DataType : int32_t {
    INVALID = 0,
    PRED = 1,
    S8 = 2,
    S16 = 3,
    S32 = 4,
    S64 = 5,
    U8 = 6,
    U16 = 7,
    U32 = 8,
    U64 = 9,
    F32 = 10,
};

inline constexpr DataType PRED = DataType::PRED;
inline constexpr DataType S8 = DataType::S8;
inline constexpr DataType S16 = DataType::S16;
inline constexpr DataType S32 = DataType::S32;
inline constexpr DataType S64 = DataType::S64;
inline constexpr DataType U8 = DataType::U8;
inline constexpr DataType U16 = DataType::U16;
inline constexpr DataType U32 = DataType::U32;
inline constexpr DataType U64 = DataType::U64;
inline constexpr DataType F32 = DataType::F32;

inline size_t ByteWidth(DataType type) {
    switch (type) {
        case DataType::PRED: case DataType::S8: case DataType::U8: return 1;
        case DataType::S16: case DataType::U16: return 2;
        case DataType::S32: case DataType::U32: case DataType::F32: return 4;
        case DataType::S64: case DataType::U64: return 8;
        default: return 0;
    }
}

// A read-only view of a buffer's extents.
struct Dimensions {
    const int64_t* data_ = nullptr;
    size_t size_ = 0;
    size_t size() const { return size_; }
    int64_t operator[](size_t k) const { return data_[k]; }
    const int64_t* begin() const { return data_; }
    const int64_t* end() const { return data_ + size_; }
};

// A device buffer as a handler sees it: data pointer, element type, extents.
// As in XLA, the extents live outside the buffer object (in the caller's
// descriptor, valid for the whole call), so a view taken from a temporary
// copy of the buffer stays valid.
class AnyBuffer {
  public:
    AnyBuffer() = default;
    AnyBuffer(void* data, DataType type, const int64_t* dims, size_t rank) : data_(data), type_(type), dims_(dims), rank_(rank) {}
    DataType element_type() const { return type_; }
    Dimensions dimensions() const { return Dimensions{dims_, rank_}; }
    size_t element_count() const {
        size_t n = 1;
        for (size_t k = 0; k < rank_; ++k) n *= static_cast<size_t>(dims_[k]);
        return n;
    }
    size_t size_bytes() const { return element_count() * ByteWidth(type_); }
    void* untyped_data() const { return data_; }

  private:
    void* data_ = nullptr;
    DataType type_ = DataType::INVALID;
    const int64_t* dims_ = nullptr;
    size_t rank_ = 0;
};

template <DataType kType> struct NativeType;
template <> struct NativeType<DataType::PRED> { using type = bool; };
template <> struct NativeType<DataType::S8> { using type = int8_t; };
template <> struct NativeType<DataType::S16> { using type = int16_t; };
template <> struct NativeType<DataType::S32> { using type = int32_t; };
template <> struct NativeType<DataType::U8> { using type = uint8_t; };
template <> struct NativeType<DataType::U32> { using type = uint32_t; };

// A buffer whose element type is fixed by the handler's signature.
template <DataType kType>
class Buffer {
  public:
    Buffer() = default;
    explicit Buffer(const AnyBuffer& any) : any_(any) {}
    Dimensions dimensions() const { return any_.dimensions(); }
    size_t element_count() const { return any_.element_count(); }
    size_t size_bytes() const { return any_.size_bytes(); }
    void* untyped_data() const { return any_.untyped_data(); }
    typename NativeType<kType>::type* typed_data() const {
        return static_cast<typename NativeType<kType>::type*>(any_.untyped_data());
    }
    DataType element_type() const { return kType; }

  private:
    AnyBuffer any_;
};

// A result buffer: dereferences to the buffer written.
template <typename T>
class Result {
  public:
    Result() = default;
    explicit Result(T value) : value_(value) {}
    T& operator*() { return value_; }
    const T& operator*() const { return value_; }
    T* operator->() { return &value_; }
    const T* operator->() const { return &value_; }

  private:
    T value_;
};

// Success or a failure with a message.
class Error {
  public:
    Error() = default;
    static Error Success() { return Error(); }
    static Error InvalidArgument(std::string message) { return Error(3, std::move(message)); }
    static Error Internal(std::string message) { return Error(13, std::move(message)); }
    bool success() const { return code_ == 0; }
    bool failure() const { return code_ != 0; }
    int code() const { return code_; }
    const std::string& message() const { return message_; }

  private:
    Error(int code, std::string message) : code_(code), message_(std::move(message)) {}
    int code_ = 0;
    std::string message_;
};

// A value or an Error.
template <typename T>
class ErrorOr {
  public:
    ErrorOr(T value) : value_(std::move(value)), ok_(true) {}
    ErrorOr(Error error) : error_(std::move(error)), ok_(false) {}
    bool has_value() const { return ok_; }
    bool has_error() const { return !ok_; }
    Error error() const { return error_; }
    T& value() { return value_; }
    const T& value() const { return value_; }
    T& operator*() { return value_; }
    const T& operator*() const { return value_; }
    T* operator->() { return &value_; }
    const T* operator->() const { return &value_; }

  private:
    T value_{};
    Error error_;
    bool ok_ = false;
};

// The operands a handler receives after its fixed arguments.
class RemainingArgs {
  public:
    RemainingArgs() = default;
    RemainingArgs(const AnyBuffer* items, size_t count) : items_(items), count_(count) {}
    size_t size() const { return count_; }
    template <typename T>
    ErrorOr<T> get(size_t index) const {
        if (index >= count_) return Error::InvalidArgument("operand index out of range");
        return T(items_[index]);
    }

  private:
    const AnyBuffer* items_ = nullptr;
    size_t count_ = 0;
};

// The results a handler writes after its fixed results.
class RemainingRets {
  public:
    RemainingRets() = default;
    RemainingRets(const AnyBuffer* items, size_t count) : items_(items), count_(count) {}
    size_t size() const { return count_; }
    template <typename T>
    ErrorOr<Result<T>> get(size_t index) const {
        if (index >= count_) return Error::InvalidArgument("result index out of range");
        return Result<T>(T(items_[index]));
    }

  private:
    const AnyBuffer* items_ = nullptr;
    size_t count_ = 0;
};

// A read-only array attribute.
template <typename T>
class Span {
  public:
    Span() = default;
    Span(T* data, size_t size) : data_(data), size_(size) {}
    T* data() const { return data_; }
    size_t size() const { return size_; }
    T& operator[](size_t k) const { return data_[k]; }
    T* begin() const { return data_; }
    T* end() const { return data_ + size_; }

  private:
    T* data_ = nullptr;
    size_t size_ = 0;
};

template <typename T>
struct PlatformStream {};

enum class Traits : uint32_t { kCmdBufferCompatible = 1 };

}  // namespace xla::ffi

// Exports the implementation's address as `<name>_implementation()`; the
// binding expression is not evaluated.
#define XLA_FFI_DEFINE_HANDLER_SYMBOL(name, implementation, binding, ...) \
    extern "C" void* name##_implementation(void) { return reinterpret_cast<void*>(&implementation); }
