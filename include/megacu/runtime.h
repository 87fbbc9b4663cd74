// Host authoring API: phases of tasks and event tensors, attributes, and the
// target runtime / dispatcher / scheduler component entry points.
//
// Interface parity with megacu `include/megacu/runtime.h:16-434`. Every public
// name, template parameter, field and error code below is kept so that an
// orchestration written against megacu (e.g. its
// `gemm_allreduce_orchestrate_common.h:24-76`) compiles unchanged:
//   progress_model, task_ref, event_tensor_ref, invalid_*_ref, attr_kind,
//   attr, attr_set (8 entries), scheduler::depends_on, events::{shape,
//   publish, acquire, join}, dispatcher::tile_grid, attrs(...),
//   operator_ref<Sig>, op(...), task_kind, linked_task, linked_event_tensor,
//   dispatcher::dispatch_state / map_explicit_attrs,
//   scheduler::{run,validate}_explicit_asap, target::{run,validate}_phase,
//   phase<Driver, MaxTasks = 64, MaxEvents = 16>, make_phase,
//   cuda_nvshmem::driver_view, cuda_nvshmem::events::{symmetric_i32_storage,
//   team_scope}.
// Error codes: phase task overflow -> invalid_argument/4, event overflow ->
// invalid_argument/5, missing operator entry -> invalid_argument/1.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <span>
#include <tuple>
#include <type_traits>
#include <utility>

#include <megacu/backends/nvshmem.h>
#include <megacu/platform/cuda.h>
#include <megacu/views.h>

namespace megacu::runtime {

enum class progress_model : std::uint8_t { asap, co_resident_persistent };

struct task_ref {
  std::uint32_t value = 0;
};

struct event_tensor_ref {
  std::uint32_t value = 0;
};

constexpr task_ref invalid_task_ref() { return {0xffffffffu}; }

constexpr event_tensor_ref invalid_event_tensor_ref() { return {0xffffffffu}; }

constexpr bool operator==(task_ref a, task_ref b) { return a.value == b.value; }

constexpr bool operator==(event_tensor_ref a, event_tensor_ref b) {
  return a.value == b.value;
}

enum class attr_kind : std::uint8_t {
  dependency,
  dispatch_tile_grid,
  event_tensor_shape,
  event_tensor_storage,
  event_tensor_scope,
  event_publish,
  event_acquire,
  event_join
};

// One typed attribute. Which fields are meaningful depends on `kind`.
struct attr {
  attr_kind kind = attr_kind::dependency;
  task_ref task;
  event_tensor_ref event;
  void *pointer = nullptr;
  std::int64_t first = 0;
  std::int64_t second = 0;
};

// Fixed-capacity list of attributes (no heap allocation).
class attr_set {
 public:
  static constexpr std::size_t max_attrs = 8;

  bool push(attr item) {
    if (count_ == max_attrs) {
      return false;
    }
    items_[count_] = item;
    ++count_;
    return true;
  }

  std::span<attr const> entries() const { return {items_.data(), count_}; }

  std::size_t size() const { return count_; }

 private:
  std::array<attr, max_attrs> items_{};
  std::size_t count_ = 0;
};

namespace scheduler {

inline attr depends_on(task_ref task) {
  attr a;
  a.kind = attr_kind::dependency;
  a.task = task;
  return a;
}

}  // namespace scheduler

namespace events {

inline attr shape(std::int64_t first, std::int64_t second) {
  attr a;
  a.kind = attr_kind::event_tensor_shape;
  a.first = first;
  a.second = second;
  return a;
}

inline attr publish(event_tensor_ref event) {
  attr a;
  a.kind = attr_kind::event_publish;
  a.event = event;
  return a;
}

inline attr acquire(event_tensor_ref event) {
  attr a;
  a.kind = attr_kind::event_acquire;
  a.event = event;
  return a;
}

inline attr join(event_tensor_ref event) {
  attr a;
  a.kind = attr_kind::event_join;
  a.event = event;
  return a;
}

}  // namespace events

namespace dispatcher {

inline attr tile_grid(std::int64_t m_tiles, std::int64_t n_tiles) {
  attr a;
  a.kind = attr_kind::dispatch_tile_grid;
  a.first = m_tiles;
  a.second = n_tiles;
  return a;
}

}  // namespace dispatcher

template <class... Items>
attr_set attrs(Items... items) {
  static_assert(sizeof...(Items) <= attr_set::max_attrs,
                "megacu attr_set capacity exceeded");
  attr_set out;
  (static_cast<void>(out.push(attr(items))), ...);
  return out;
}

// A named native operator with a fixed signature.
template <class Signature>
struct operator_ref;

template <class R, class... Args>
struct operator_ref<R(Args...)> {
  using function_type = R(Args...);
  using return_type = R;
  static constexpr std::size_t arity = sizeof...(Args);

  char const *name = nullptr;
  function_type *entry = nullptr;
};

template <class R, class... Args>
operator_ref<R(Args...)> op(char const *name, R (*entry)(Args...)) {
  operator_ref<R(Args...)> ref;
  ref.name = name;
  ref.entry = entry;
  return ref;
}

template <class Signature>
operator_ref<Signature> op(char const *name) {
  operator_ref<Signature> ref;
  ref.name = name;
  return ref;
}

enum class task_kind : std::uint8_t { operator_body, sync_only };

struct linked_task {
  task_kind kind = task_kind::operator_body;
  char const *op_name = nullptr;
  std::uint16_t raw_arg_count = 0;
  attr_set attributes;
  std::function<status()> invoke;
};

struct linked_event_tensor {
  event_tensor_ref ref;
  attr_set attributes;
};

namespace dispatcher {

// Counts the dispatcher derives from a phase's attributes.
struct dispatch_state {
  std::size_t task_count = 0;
  std::size_t event_tensor_count = 0;
  std::int64_t tile_grid_attrs = 0;
  std::int64_t total_tile_count = 0;
  std::int64_t sync_task_count = 0;
  std::int64_t sync_event_count = 0;
  std::int64_t event_publish_attrs = 0;
  std::int64_t event_acquire_attrs = 0;
  std::int64_t event_join_attrs = 0;
};

status map_explicit_attrs(dispatch_state &out,
                          std::span<linked_task const> tasks,
                          std::span<linked_event_tensor const> events = {});

}  // namespace dispatcher

namespace scheduler {

status run_explicit_asap(std::span<linked_task const> tasks,
                         dispatcher::dispatch_state const &dispatch,
                         progress_model progress);

status validate_explicit_asap(std::span<linked_task const> tasks,
                              dispatcher::dispatch_state const &dispatch,
                              progress_model progress);

}  // namespace scheduler

namespace target {

status run_phase(std::span<linked_task const> tasks,
                 std::span<linked_event_tensor const> events,
                 progress_model progress);

status validate_phase(std::span<linked_task const> tasks,
                      std::span<linked_event_tensor const> events,
                      progress_model progress);

}  // namespace target

namespace detail {

// Arguments passed to submit()/run() are the operator's raw arguments,
// optionally followed by one attr_set.
template <class... Ts>
struct ends_with_attrs : std::false_type {};

template <class T, class... Ts>
struct ends_with_attrs<T, Ts...>
    : std::is_same<std::remove_cvref_t<
                       std::tuple_element_t<sizeof...(Ts),
                                            std::tuple<T, Ts...>>>,
                   attr_set> {};

template <class... Ts>
inline constexpr std::size_t raw_arg_count_v =
    sizeof...(Ts) - (ends_with_attrs<Ts...>::value ? 1 : 0);

template <class... Ts>
attr_set trailing_attrs(Ts &&...items) {
  if constexpr (ends_with_attrs<Ts...>::value) {
    return std::get<sizeof...(Ts) - 1>(std::forward_as_tuple(items...));
  } else {
    return {};
  }
}

template <class... Ts, std::size_t... I>
auto copy_leading(std::tuple<Ts...> const &all, std::index_sequence<I...>) {
  return std::make_tuple(std::decay_t<std::tuple_element_t<I, std::tuple<Ts...>>>(
      std::get<I>(all))...);
}

template <std::size_t N, class... Ts>
auto leading_args(Ts &&...items) {
  return copy_leading(std::forward_as_tuple(items...),
                      std::make_index_sequence<N>{});
}

template <class R, class Fn, class Tuple>
status invoke_as_status(Fn *fn, Tuple &args) {
  if (fn == nullptr) {
    return {status_code::invalid_argument, 1, "missing operator entry"};
  }
  if constexpr (std::is_same_v<R, status>) {
    return std::apply(fn, args);
  } else {
    std::apply(fn, args);
    return {};
  }
}

}  // namespace detail

// A phase records tasks (native operators or sync points) and event tensors,
// then either runs the operator tasks on the host in ASAP order (`run()`) or
// validates the graph and hands the whole phase to one native launcher
// (`run(launcher, args...)`), which is how the megakernel is entered.
template <class Driver, std::size_t MaxTasks = 64, std::size_t MaxEvents = 16>
class phase {
 public:
  phase(Driver &driver, progress_model progress)
      : driver_(&driver), progress_(progress) {}

  event_tensor_ref event_tensor(attr_set attributes = {}) {
    if (latched_.code != status_code::ok || n_events_ == MaxEvents) {
      latched_ = {status_code::invalid_argument, 5,
                  "megacu event tensor capacity exceeded"};
      return invalid_event_tensor_ref();
    }
    event_tensor_ref ref{static_cast<std::uint32_t>(n_events_)};
    events_[n_events_].ref = ref;
    events_[n_events_].attributes = attributes;
    ++n_events_;
    return ref;
  }

  template <class Signature, class... Submitted>
  task_ref submit(operator_ref<Signature> op, Submitted &&...submitted) {
    constexpr std::size_t n_raw = detail::raw_arg_count_v<Submitted...>;
    static_assert(n_raw == operator_ref<Signature>::arity,
                  "megacu task args must match the native operator "
                  "signature; pass optional runtime attrs as the final "
                  "argument");
    if (latched_.code != status_code::ok || n_tasks_ == MaxTasks) {
      latched_ = {status_code::invalid_argument, 4,
                  "megacu phase task capacity exceeded"};
      return invalid_task_ref();
    }
    auto args = detail::leading_args<n_raw>(submitted...);
    linked_task &task = tasks_[n_tasks_];
    task.kind = task_kind::operator_body;
    task.op_name = op.name;
    task.raw_arg_count = static_cast<std::uint16_t>(n_raw);
    task.attributes = detail::trailing_attrs(submitted...);
    task.invoke = [fn = op.entry, args]() mutable -> status {
      using R = typename operator_ref<Signature>::return_type;
      return detail::invoke_as_status<R>(fn, args);
    };
    return task_ref{static_cast<std::uint32_t>(n_tasks_++)};
  }

  task_ref sync(attr_set attributes = {}) {
    if (latched_.code != status_code::ok || n_tasks_ == MaxTasks) {
      latched_ = {status_code::invalid_argument, 4,
                  "megacu phase task capacity exceeded"};
      return invalid_task_ref();
    }
    linked_task &task = tasks_[n_tasks_];
    task.kind = task_kind::sync_only;
    task.op_name = "sync";
    task.raw_arg_count = 0;
    task.attributes = attributes;
    task.invoke = nullptr;
    return task_ref{static_cast<std::uint32_t>(n_tasks_++)};
  }

  // Runs the operator tasks on the host in ASAP order.
  status run() {
    if (latched_.code != status_code::ok) {
      return latched_;
    }
    return target::run_phase(tasks(), event_tensors(), progress_);
  }

  // Validates the phase, then calls only `launcher` with `submitted...`.
  template <class Signature, class... Submitted>
  status run(operator_ref<Signature> launcher, Submitted &&...submitted) {
    constexpr std::size_t n_raw = detail::raw_arg_count_v<Submitted...>;
    static_assert(n_raw == operator_ref<Signature>::arity,
                  "megacu launcher args must match the native launcher "
                  "signature");
    if (latched_.code != status_code::ok) {
      return latched_;
    }
    status checked = target::validate_phase(tasks(), event_tensors(), progress_);
    if (checked.code != status_code::ok) {
      return checked;
    }
    auto args = detail::leading_args<n_raw>(submitted...);
    using R = typename operator_ref<Signature>::return_type;
    return detail::invoke_as_status<R>(launcher.entry, args);
  }

  Driver &driver() const { return *driver_; }

  progress_model progress() const { return progress_; }

  std::span<linked_task const> tasks() const { return {tasks_.data(), n_tasks_}; }

  std::span<linked_event_tensor const> event_tensors() const {
    return {events_.data(), n_events_};
  }

 private:
  Driver *driver_ = nullptr;
  progress_model progress_ = progress_model::asap;
  std::array<linked_task, MaxTasks> tasks_{};
  std::array<linked_event_tensor, MaxEvents> events_{};
  std::size_t n_tasks_ = 0;
  std::size_t n_events_ = 0;
  status latched_;
};

template <class Driver>
phase<Driver> make_phase(Driver &driver, progress_model progress) {
  return phase<Driver>(driver, progress);
}

}  // namespace megacu::runtime

namespace megacu::cuda_nvshmem {

struct driver_view {
  megacu::cuda::launch_view launch;
  megacu::nvshmem::team_view team;
};

namespace events {

inline megacu::runtime::attr symmetric_i32_storage(void *storage) {
  megacu::runtime::attr a;
  a.kind = megacu::runtime::attr_kind::event_tensor_storage;
  a.pointer = storage;
  return a;
}

inline megacu::runtime::attr team_scope() {
  megacu::runtime::attr a;
  a.kind = megacu::runtime::attr_kind::event_tensor_scope;
  return a;
}

}  // namespace events

}  // namespace megacu::cuda_nvshmem
