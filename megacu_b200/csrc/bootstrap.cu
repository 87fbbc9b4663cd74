// Launch adapter: team set-up for processes on one node without MPI,
// NVSHMEM's launcher or torch.distributed (a B200 addition).
//
// megacu sets its team up with nvshmem_init under an NVSHMEM launcher and
// lists MPI / torch adapters as future work. Here the handle exchange that
// megacu_b200_team_connect needs can run over an abstract unix socket named
// by a session string every PE is given (the role NVSHMEM's unique id plays
// in a uid bootstrap): PE 0 listens, every other PE connects and sends its
// blob, PE 0 answers each with every blob in PE order. Every wait is bounded
// by the caller's timeout; a missing, late or duplicate PE ends the exchange
// with MEGACU_BACKEND_ERROR / detail 39 on the PEs that notice it.
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

#include <megacu_b200.h>

namespace {

constexpr std::uint32_t kMagic = 0x6d633278u;  // "mc2x"
constexpr std::size_t kMaxSession = 64;

using clock_type = std::chrono::steady_clock;

megacu_status ok_status() { return {MEGACU_OK, 0, nullptr}; }

megacu_status fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

megacu_status exchange_fail(char const *msg) { return fail(MEGACU_BACKEND_ERROR, 39, msg); }

struct header {
  std::uint32_t magic;
  std::int32_t pe;
  std::int64_t bytes;
};

bool session_address(char const *session, sockaddr_un &addr, socklen_t &len) {
  char const prefix[] = "megacu_b200.x.";
  std::size_t const n = std::strlen(session);
  std::size_t const total = sizeof(prefix) - 1 + n;
  std::memset(&addr, 0, sizeof(addr));
  addr.sun_family = AF_UNIX;
  if (total + 1 > sizeof(addr.sun_path)) return false;
  std::memcpy(addr.sun_path + 1, prefix, sizeof(prefix) - 1);  // sun_path[0] = 0: abstract
  std::memcpy(addr.sun_path + 1 + sizeof(prefix) - 1, session, n);
  len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + total);
  return true;
}

int ms_left(clock_type::time_point deadline) {
  auto const left =
      std::chrono::duration_cast<std::chrono::milliseconds>(deadline - clock_type::now()).count();
  return left > 0 ? static_cast<int>(left) : 0;
}

// Moves exactly `n` bytes (recv or send) before the deadline.
bool transfer(int fd, void *buf, std::size_t n, bool sending, clock_type::time_point deadline) {
  auto *p = static_cast<char *>(buf);
  while (n > 0) {
    pollfd pfd{fd, static_cast<short>(sending ? POLLOUT : POLLIN), 0};
    int const wait = ms_left(deadline);
    if (wait == 0 || poll(&pfd, 1, wait) <= 0) return false;
    ssize_t const r = sending ? send(fd, p, n, MSG_NOSIGNAL) : recv(fd, p, n, 0);
    if (r <= 0) return false;
    p += r;
    n -= static_cast<std::size_t>(r);
  }
  return true;
}

megacu_status serve(sockaddr_un const &addr, socklen_t len, std::int32_t n_pes,
                    std::int64_t bytes, void const *mine, void *all,
                    clock_type::time_point deadline) {
  int const s = socket(AF_UNIX, SOCK_STREAM, 0);
  if (s < 0) return exchange_fail("cannot open the rendezvous socket");
  if (bind(s, reinterpret_cast<sockaddr const *>(&addr), len) != 0 || listen(s, n_pes) != 0) {
    close(s);
    return exchange_fail("cannot listen on the rendezvous socket (session in use?)");
  }
  auto *out = static_cast<char *>(all);
  std::memcpy(out, mine, static_cast<std::size_t>(bytes));
  std::vector<int> clients(static_cast<std::size_t>(n_pes), -1);
  std::int32_t joined = 1;
  megacu_status st = ok_status();
  while (joined < n_pes) {
    pollfd pfd{s, POLLIN, 0};
    int const wait = ms_left(deadline);
    if (wait == 0 || poll(&pfd, 1, wait) <= 0) {
      st = exchange_fail("not every PE joined the rendezvous in time");
      break;
    }
    int const c = accept(s, nullptr, nullptr);
    if (c < 0) continue;
    header h{};
    if (!transfer(c, &h, sizeof(h), false, deadline) || h.magic != kMagic || h.bytes != bytes ||
        h.pe <= 0 || h.pe >= n_pes || clients[h.pe] >= 0) {
      close(c);
      st = exchange_fail("a PE joined the rendezvous with a bad, duplicate or mismatched blob");
      break;
    }
    if (!transfer(c, out + h.pe * bytes, static_cast<std::size_t>(bytes), false, deadline)) {
      close(c);
      st = exchange_fail("a PE's blob did not arrive in time");
      break;
    }
    clients[h.pe] = c;
    ++joined;
  }
  close(s);
  std::size_t const total = static_cast<std::size_t>(n_pes) * static_cast<std::size_t>(bytes);
  for (std::int32_t pe = 1; pe < n_pes; ++pe) {
    int const c = clients[pe];
    if (c < 0) continue;
    // On failure the clients get nothing and report it themselves.
    if (st.code == MEGACU_OK && !transfer(c, out, total, true, deadline)) {
      st = exchange_fail("could not send every blob back to a PE");
    }
    close(c);
  }
  return st;
}

megacu_status join(sockaddr_un const &addr, socklen_t len, std::int32_t my_pe,
                   std::int32_t n_pes, std::int64_t bytes, void const *mine, void *all,
                   clock_type::time_point deadline) {
  int s = -1;
  for (;;) {
    s = socket(AF_UNIX, SOCK_STREAM, 0);
    if (s < 0) return exchange_fail("cannot open the rendezvous socket");
    if (connect(s, reinterpret_cast<sockaddr const *>(&addr), len) == 0) break;
    close(s);
    s = -1;
    if (ms_left(deadline) == 0) return exchange_fail("PE 0 did not open the rendezvous in time");
    usleep(5000);
  }
  header h{kMagic, my_pe, bytes};
  std::size_t const total = static_cast<std::size_t>(n_pes) * static_cast<std::size_t>(bytes);
  bool const ok = transfer(s, &h, sizeof(h), true, deadline) &&
                  transfer(s, const_cast<void *>(mine), static_cast<std::size_t>(bytes), true,
                           deadline) &&
                  transfer(s, all, total, false, deadline);
  close(s);
  return ok ? ok_status() : exchange_fail("the rendezvous ended before every blob arrived");
}

}  // namespace

extern "C" megacu_status megacu_b200_exchange_local(char const *session, std::int32_t my_pe,
                                                    std::int32_t n_pes, void const *mine,
                                                    std::int64_t bytes, void *all,
                                                    std::int64_t timeout_ms) {
  if (session == nullptr || mine == nullptr || all == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  std::size_t const n = std::strlen(session);
  if (n == 0 || n > kMaxSession || bytes <= 0 || bytes > (std::int64_t(1) << 30) ||
      timeout_ms <= 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "session must be 1-64 characters, bytes and timeout > 0");
  }
  if (n_pes < 1 || n_pes > 1024 || my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team size / PE index out of range");
  }
  if (n_pes == 1) {
    std::memcpy(all, mine, static_cast<std::size_t>(bytes));
    return ok_status();
  }
  sockaddr_un addr;
  socklen_t len;
  if (!session_address(session, addr, len)) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "session name too long");
  }
  auto const deadline = clock_type::now() + std::chrono::milliseconds(timeout_ms);
  return my_pe == 0 ? serve(addr, len, n_pes, bytes, mine, all, deadline)
                    : join(addr, len, my_pe, n_pes, bytes, mine, all, deadline);
}

extern "C" megacu_status megacu_b200_team_create_local(char const *session, std::int32_t my_pe,
                                                       std::int32_t n_pes, std::int32_t device,
                                                       std::int64_t heap_bytes,
                                                       std::int64_t timeout_ms, void **team) {
  if (team == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  *team = nullptr;
  void *t = nullptr;
  megacu_status st = megacu_b200_team_create(my_pe, n_pes, device, heap_bytes, &t);
  if (st.code != MEGACU_OK) return st;
  if (n_pes > 1) {
    std::vector<unsigned char> mine(MEGACU_B200_TEAM_HANDLE_BYTES);
    std::vector<unsigned char> all(static_cast<std::size_t>(n_pes) * MEGACU_B200_TEAM_HANDLE_BYTES);
    st = megacu_b200_team_export(t, mine.data());
    if (st.code == MEGACU_OK) {
      st = megacu_b200_exchange_local(session, my_pe, n_pes, mine.data(),
                                      MEGACU_B200_TEAM_HANDLE_BYTES, all.data(), timeout_ms);
    }
    if (st.code == MEGACU_OK) st = megacu_b200_team_connect(t, all.data());
    if (st.code != MEGACU_OK) {
      megacu_b200_team_destroy(t);
      return st;
    }
  }
  *team = t;
  return ok_status();
}
