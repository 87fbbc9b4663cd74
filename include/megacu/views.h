// Core value types shared by the host runtime, the C ABI and the device code.
//
// Interface parity: the enum values, struct fields and their order are the
// ABI of megacu's `include/megacu/views.h:12-61` (dtype, status_code, status,
// backend/session ids, buffer and tensor views). They are kept identical so
// that code written against megacu compiles and links against this library
// unchanged, and so that `megacu::status` returned by value from the
// `extern "C"` launchers has the same layout as the reference's.
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>

namespace megacu {

template <class T, std::size_t Extent = std::dynamic_extent>
using span = std::span<T, Extent>;

// Element type of a tensor. Numbering follows megacu (views.h:12-17).
enum class dtype : std::uint16_t { unknown = 0, f16, bf16, f32 };

// Error class of a `status`. Numbering follows megacu (views.h:19-25).
enum class status_code : std::uint8_t {
  ok,
  invalid_argument,
  unsupported,
  backend_error,
  launch_error
};

// Result of every runtime call. `detail` is a per-call-site number,
// `message` a static string (or a CUDA error string). Nothing throws.
struct status {
  status_code code = status_code::ok;
  std::uint16_t detail = 0;
  char const *message = nullptr;
};

struct backend_id {
  std::uint16_t value = 0;
};

struct session_id {
  std::uint64_t value = 0;
};

// A buffer that lives at the same offset of every rank's symmetric heap.
struct symmetric_buffer_view {
  void *data = nullptr;
  std::int64_t bytes = 0;
  backend_id backend;
  session_id session;
};

struct event_storage_view {
  symmetric_buffer_view buffer;
};

struct tensor_view {
  void *data = nullptr;
  std::int64_t bytes = 0;
  dtype type = dtype::unknown;
};

struct symmetric_tensor_view {
  symmetric_buffer_view buffer;
  dtype type = dtype::unknown;
};

}  // namespace megacu
