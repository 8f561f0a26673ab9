// Stand-in for jaxlib's xla/ffi/api/ffi.h, used to compile and test the
// codec's XLA FFI handlers (ffi/cuda_zlib_xla.cc) where jaxlib is not
// installed.  It declares the part of the typed FFI API the handlers use,
// with the same names and member functions: Buffer<T> (typed_data,
// element_count, dimensions), ResultBuffer<T>, Span<T>, Error,
// PlatformStream<T> and the Ffi::Bind() builder.
//
// XLA_FFI_DEFINE_HANDLER_SYMBOL checks the handler against its binding at
// compile time and exports an extern "C" function of the handler's name.
// That function decodes a call frame of this stand-in's own plain layout
// (XLA_FFI_CallFrame below, NOT XLA's C API layout), so tests can call the
// handlers through ctypes; in a JAX build, jaxlib's header replaces all of
// this and XLA passes its own call frames.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <tuple>
#include <type_traits>
#include <utility>

// ------------------------------------------------------------------ frame
extern "C" {
typedef struct XLA_FFI_StandinBuffer {
  void* data;
  int64_t rank;
  const int64_t* dims;
} XLA_FFI_StandinBuffer;

typedef struct XLA_FFI_StandinSpan {
  const int64_t* data;
  int64_t size;
} XLA_FFI_StandinSpan;

// attrs[i] points to an int64_t (scalar attribute) or an XLA_FFI_StandinSpan.
typedef struct XLA_FFI_CallFrame {
  void* stream;
  int64_t num_attrs;
  const void* const* attrs;
  int64_t num_args;
  const XLA_FFI_StandinBuffer* args;
  int64_t num_rets;
  const XLA_FFI_StandinBuffer* rets;
} XLA_FFI_CallFrame;

// Error codes follow absl::StatusCode (INVALID_ARGUMENT 3, INTERNAL 13).
typedef struct XLA_FFI_Error {
  int code;
  char message[256];
} XLA_FFI_Error;
}

namespace xla {
namespace ffi {

enum class DataType : uint8_t { U8 = 6, U32 = 8 };
inline constexpr DataType U8 = DataType::U8;
inline constexpr DataType U32 = DataType::U32;

template <DataType T> struct NativeType;
template <> struct NativeType<DataType::U8> { using type = uint8_t; };
template <> struct NativeType<DataType::U32> { using type = uint32_t; };

template <typename T>
class Span {
 public:
  Span() = default;
  Span(T* data, size_t size) : data_(data), size_(size) {}
  T* begin() const { return data_; }
  T* end() const { return data_ + size_; }
  size_t size() const { return size_; }
  T& operator[](size_t i) const { return data_[i]; }

 private:
  T* data_ = nullptr;
  size_t size_ = 0;
};

class Error {
 public:
  Error() = default;
  static Error Success() { return Error(); }
  static Error InvalidArgument(std::string message) { return Error(3, std::move(message)); }
  static Error Internal(std::string message) { return Error(13, std::move(message)); }
  bool success() const { return code_ == 0; }
  int code() const { return code_; }
  const std::string& message() const { return message_; }

 private:
  Error(int code, std::string message) : code_(code), message_(std::move(message)) {}
  int code_ = 0;
  std::string message_;
};

template <DataType T>
class Buffer {
 public:
  using Native = typename NativeType<T>::type;
  Buffer() = default;
  explicit Buffer(const XLA_FFI_StandinBuffer& b)
      : data_(static_cast<Native*>(b.data)), dims_(b.dims, size_t(b.rank)) {}
  Native* typed_data() const { return data_; }
  Span<const int64_t> dimensions() const { return dims_; }
  size_t element_count() const {
    size_t n = 1;
    for (int64_t d : dims_) n *= size_t(d);
    return n;
  }

 private:
  Native* data_ = nullptr;
  Span<const int64_t> dims_;
};

template <typename T>
class Result {
 public:
  explicit Result(T value) : value_(value) {}
  T* operator->() { return &value_; }
  const T* operator->() const { return &value_; }
  T& operator*() { return value_; }

 private:
  T value_;
};

template <DataType T>
using ResultBuffer = Result<Buffer<T>>;

template <typename T>
struct PlatformStream {};

namespace standin {
// Binding slots, in declaration order.
template <typename T> struct CtxSlot { using type = T; };
template <typename T> struct AttrSlot { using type = T; };
template <typename T> struct ArgSlot { using type = T; };
template <typename T> struct RetSlot { using type = Result<T>; };

struct Cursor {
  size_t attr = 0, arg = 0, ret = 0;
};

template <typename Slot> struct Decode;
template <typename S> struct Decode<CtxSlot<PlatformStream<S>>> {
  static S get(const XLA_FFI_CallFrame* f, Cursor&) { return static_cast<S>(f->stream); }
};
template <> struct Decode<AttrSlot<int64_t>> {
  static int64_t get(const XLA_FFI_CallFrame* f, Cursor& c) {
    return *static_cast<const int64_t*>(f->attrs[c.attr++]);
  }
};
template <> struct Decode<AttrSlot<Span<const int64_t>>> {
  static Span<const int64_t> get(const XLA_FFI_CallFrame* f, Cursor& c) {
    const auto* s = static_cast<const XLA_FFI_StandinSpan*>(f->attrs[c.attr++]);
    return Span<const int64_t>(s->data, size_t(s->size));
  }
};
template <DataType T> struct Decode<ArgSlot<Buffer<T>>> {
  static Buffer<T> get(const XLA_FFI_CallFrame* f, Cursor& c) { return Buffer<T>(f->args[c.arg++]); }
};
template <DataType T> struct Decode<RetSlot<Buffer<T>>> {
  static Result<Buffer<T>> get(const XLA_FFI_CallFrame* f, Cursor& c) {
    return Result<Buffer<T>>(Buffer<T>(f->rets[c.ret++]));
  }
};

template <typename... Slots>
struct Binding {
  template <typename T> Binding<Slots..., CtxSlot<T>> Ctx() const { return {}; }
  template <typename T> Binding<Slots..., AttrSlot<T>> Attr(const char*) const { return {}; }
  template <typename T> Binding<Slots..., ArgSlot<T>> Arg() const { return {}; }
  template <typename T> Binding<Slots..., RetSlot<T>> Ret() const { return {}; }

  // Decodes the frame in slot order (braced initialisation is sequenced)
  // and calls the handler.
  template <typename Fn>
  static Error Call(Fn&& fn, const XLA_FFI_CallFrame* frame) {
    Cursor cursor;
    std::tuple<decltype(Decode<Slots>::get(frame, cursor))...> values{
        Decode<Slots>::get(frame, cursor)...};
    return std::apply(fn, std::move(values));
  }

  template <typename Fn>
  static constexpr bool Accepts() {
    return std::is_invocable_r_v<Error, Fn,
                                 decltype(Decode<Slots>::get(nullptr, std::declval<Cursor&>()))...>;
  }
};

inline XLA_FFI_Error* Report(const Error& e) {
  if (e.success()) return nullptr;
  static thread_local XLA_FFI_Error record;
  record.code = e.code();
  const size_t n = e.message().size() < sizeof(record.message) - 1 ? e.message().size()
                                                                     : sizeof(record.message) - 1;
  e.message().copy(record.message, n);
  record.message[n] = 0;
  return &record;
}
}  // namespace standin

struct Ffi {
  static standin::Binding<> Bind() { return {}; }
};

}  // namespace ffi
}  // namespace xla

#define XLA_FFI_DEFINE_HANDLER_SYMBOL(fn, impl, binding)                               \
  static_assert(std::decay_t<decltype(binding)>::template Accepts<decltype(&impl)>(), \
                #impl " does not match the binding of " #fn);                         \
  extern "C" __attribute__((visibility("default"))) XLA_FFI_Error* fn(                 \
      XLA_FFI_CallFrame* frame) {                                                      \
    try {                                                                              \
      return ::xla::ffi::standin::Report(                                              \
          std::decay_t<decltype(binding)>::Call(impl, frame));                         \
    } catch (...) {                                                                    \
      return ::xla::ffi::standin::Report(                                              \
          ::xla::ffi::Error::Internal("stand-in frame decoding failed"));              \
    }                                                                                  \
  }
