// Native host transport: a full mesh of TCP connections between ranks.
//
// Host-side counterpart of the reference's pure-Python transport
// (mini_nccl/transport.py:1-216, mini_nccl/process_group.py:95-148).  The wire
// contract is the same (raw bytes, no framing, both ends agree on sizes), but
// the mechanics are native:
//
//   * rendezvous: rank r listens on addrs[r]; a poll()-driven acceptor thread
//     takes connections from higher ranks while this thread dials every lower
//     rank with retries.  A 12-byte hello (magic, rank, channel) identifies
//     each dialled socket.  A failed rendezvous stops the acceptor, closes the
//     listener and every half-built connection, so a retry can rebind.
//   * full-duplex exchange runs in ONE thread with non-blocking sockets and
//     poll(): the send to `dst` and the receive from `src` both make progress
//     in the same loop, so ring steps cannot deadlock and no helper thread is
//     needed per channel.
//   * every blocking wait is bounded by the op timeout, measured as time
//     without progress; expiry raises TransportTimeout, a 0-byte read raises
//     TransportPeerClosed.
//
// All blocking calls release the GIL.
#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/types.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;

namespace mnb {

struct TransportTimeout : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct TransportPeerClosed : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct TransportRendezvous : std::runtime_error {
  using std::runtime_error::runtime_error;
};

namespace {

constexpr uint32_t kHelloMagic = 0x4d4e4232u;  // "MNB2"
constexpr int kSockBuf = 4 << 20;
constexpr int kAcceptPollMs = 100;

using Clock = std::chrono::steady_clock;

double seconds_since(Clock::time_point t0) {
  return std::chrono::duration<double>(Clock::now() - t0).count();
}

void set_nonblocking(int fd, bool on) {
  int flags = fcntl(fd, F_GETFL, 0);
  if (on)
    flags |= O_NONBLOCK;
  else
    flags &= ~O_NONBLOCK;
  fcntl(fd, F_SETFL, flags);
}

void tune_socket(int fd) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  int buf = kSockBuf;
  setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &buf, sizeof(buf));
  setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &buf, sizeof(buf));
}

bool resolve(const std::string& host, int port, sockaddr_storage* out, socklen_t* len) {
  addrinfo hints{};
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  addrinfo* res = nullptr;
  std::string port_s = std::to_string(port);
  if (getaddrinfo(host.c_str(), port_s.c_str(), &hints, &res) != 0 || res == nullptr) return false;
  std::memcpy(out, res->ai_addr, res->ai_addrlen);
  *len = res->ai_addrlen;
  freeaddrinfo(res);
  return true;
}

// Blocking-style full read/write used only during the handshake, bounded by
// a deadline so a half-open peer cannot wedge rendezvous.
bool io_all(int fd, char* buf, size_t n, bool is_write, double timeout_s) {
  auto t0 = Clock::now();
  size_t done = 0;
  while (done < n) {
    pollfd p{fd, static_cast<short>(is_write ? POLLOUT : POLLIN), 0};
    int left_ms = static_cast<int>((timeout_s - seconds_since(t0)) * 1000);
    if (left_ms <= 0) return false;
    int rc = poll(&p, 1, left_ms);
    if (rc < 0 && errno == EINTR) continue;
    if (rc <= 0) return false;
    ssize_t k = is_write ? ::send(fd, buf + done, n - done, MSG_NOSIGNAL | MSG_DONTWAIT)
                         : ::recv(fd, buf + done, n - done, MSG_DONTWAIT);
    if (k < 0 && (errno == EAGAIN || errno == EWOULDBLOCK || errno == EINTR)) continue;
    if (k <= 0) return false;
    done += static_cast<size_t>(k);
  }
  return true;
}

}  // namespace

class TcpMesh {
 public:
  TcpMesh(int rank, int world_size, std::vector<std::pair<std::string, int>> addrs, int n_channels,
          double timeout_s, double op_timeout_s)
      : rank_(rank), world_(world_size), n_channels_(n_channels), op_timeout_(op_timeout_s) {
    if (world_size < 1 || rank < 0 || rank >= world_size)
      throw std::invalid_argument("rank out of range");
    if (n_channels < 1) throw std::invalid_argument("n_channels must be >= 1");
    fds_.assign(static_cast<size_t>(world_) * n_channels_, -1);
    if (world_ == 1) return;
    if (static_cast<int>(addrs.size()) != world_)
      throw std::invalid_argument("need one (host, port) address per rank");
    py::gil_scoped_release nogil;
    rendezvous(addrs, timeout_s);
  }

  ~TcpMesh() { close(); }

  int rank() const { return rank_; }
  int world_size() const { return world_; }
  int n_channels() const { return n_channels_; }

  void set_op_timeout(double s) { op_timeout_.store(s); }
  double op_timeout() const { return op_timeout_.load(); }

  void send(int peer, int channel, uintptr_t ptr, int64_t nbytes) {
    int fd = fd_for(peer, channel);
    py::gil_scoped_release nogil;
    duplex(fd, reinterpret_cast<const char*>(ptr), nbytes, -1, nullptr, 0, 0, nullptr, peer, -1, channel);
  }

  void recv(int peer, int channel, uintptr_t ptr, int64_t nbytes) {
    int fd = fd_for(peer, channel);
    py::gil_scoped_release nogil;
    duplex(-1, nullptr, 0, fd, reinterpret_cast<char*>(ptr), nbytes, 0, nullptr, -1, peer, channel);
  }

  // Send `sn` bytes to `dst` while receiving `rn` bytes from `src`.  With
  // slice_bytes > 0 and a callback, the callback runs (GIL held) with the
  // byte range [start, end) of each receive slice as soon as it has landed.
  void exchange(int dst, uintptr_t sptr, int64_t sn, int src, uintptr_t rptr, int64_t rn,
                int channel, int64_t slice_bytes, py::object on_slice) {
    int sfd = fd_for(dst, channel);
    int rfd = fd_for(src, channel);
    std::function<void(int64_t, int64_t)> cb;
    if (!on_slice.is_none()) {
      cb = [&on_slice](int64_t a, int64_t b) {
        py::gil_scoped_acquire gil;
        on_slice(a, b);
      };
    }
    py::gil_scoped_release nogil;
    duplex(sfd, reinterpret_cast<const char*>(sptr), sn, rfd, reinterpret_cast<char*>(rptr), rn,
           slice_bytes, cb ? &cb : nullptr, dst, src, channel);
  }

  void close() {
    std::lock_guard<std::mutex> g(close_mu_);
    for (int& fd : fds_) {
      if (fd >= 0) {
        ::shutdown(fd, SHUT_RDWR);
        ::close(fd);
        fd = -1;
      }
    }
  }

 private:
  int fd_for(int peer, int channel) const {
    if (peer < 0 || peer >= world_ || peer == rank_)
      throw std::invalid_argument("invalid peer " + std::to_string(peer));
    if (channel < 0 || channel >= n_channels_)
      throw std::invalid_argument("invalid channel " + std::to_string(channel));
    int fd = fds_[static_cast<size_t>(peer) * n_channels_ + channel];
    if (fd < 0) throw TransportPeerClosed("connection is closed");
    return fd;
  }

  // The one progress engine behind send, recv and exchange.
  void duplex(int sfd, const char* sbuf, int64_t sn, int rfd, char* rbuf, int64_t rn,
              int64_t slice_bytes, std::function<void(int64_t, int64_t)>* cb, int dst, int src,
              int channel) {
    int64_t sent = 0, got = 0, reported = 0;
    auto last_progress = Clock::now();
    while (sent < sn || got < rn) {
      pollfd pf[2];
      int np = 0;
      int si = -1, ri = -1;
      if (sent < sn && sfd >= 0) {
        pf[np] = {sfd, POLLOUT, 0};
        si = np++;
      }
      if (got < rn && rfd >= 0) {
        if (si >= 0 && pf[si].fd == rfd) {
          pf[si].events |= POLLIN;
          ri = si;
        } else {
          pf[np] = {rfd, POLLIN, 0};
          ri = np++;
        }
      }
      double limit = op_timeout_.load();
      int wait_ms = 200;
      int rc = poll(pf, np, wait_ms);
      if (rc < 0) {
        if (errno == EINTR) continue;
        throw std::runtime_error(std::string("poll failed: ") + std::strerror(errno));
      }
      bool progressed = false;
      if (si >= 0 && (pf[si].revents & (POLLOUT | POLLERR | POLLHUP))) {
        ssize_t k = ::send(sfd, sbuf + sent, static_cast<size_t>(sn - sent), MSG_NOSIGNAL | MSG_DONTWAIT);
        if (k > 0) {
          sent += k;
          progressed = true;
        } else if (k < 0 && errno != EAGAIN && errno != EWOULDBLOCK && errno != EINTR) {
          throw TransportPeerClosed("send to rank " + std::to_string(dst) + " on channel " +
                                    std::to_string(channel) + " failed: " + std::strerror(errno));
        }
      }
      if (ri >= 0 && (pf[ri].revents & (POLLIN | POLLERR | POLLHUP))) {
        ssize_t k = ::recv(rfd, rbuf + got, static_cast<size_t>(rn - got), MSG_DONTWAIT);
        if (k > 0) {
          got += k;
          progressed = true;
        } else if (k == 0) {
          throw TransportPeerClosed("rank " + std::to_string(src) + " closed channel " +
                                    std::to_string(channel) + " mid-message");
        } else if (errno != EAGAIN && errno != EWOULDBLOCK && errno != EINTR) {
          throw TransportPeerClosed("recv from rank " + std::to_string(src) + " failed: " +
                                    std::strerror(errno));
        }
      }
      if (cb && got > reported) {
        int64_t step = slice_bytes > 0 ? slice_bytes : rn;
        while (reported < got && (got - reported >= step || got == rn)) {
          int64_t end = std::min(rn, reported + step);
          if (end > got) break;
          (*cb)(reported, end);
          reported = end;
        }
      }
      if (progressed) {
        last_progress = Clock::now();
      } else if (limit > 0 && seconds_since(last_progress) > limit) {
        std::ostringstream os;
        os << "no progress for " << limit << "s (sent " << sent << "/" << sn << " to rank " << dst
           << ", received " << got << "/" << rn << " from rank " << src << ", channel " << channel
           << ")";
        throw TransportTimeout(os.str());
      }
    }
    if (cb && reported < rn) (*cb)(reported, rn);
  }

  void rendezvous(const std::vector<std::pair<std::string, int>>& addrs, double timeout_s) {
    sockaddr_storage sa{};
    socklen_t salen = 0;
    const auto& me = addrs[rank_];
    if (!resolve(me.first, me.second, &sa, &salen))
      throw TransportRendezvous("rank " + std::to_string(rank_) + ": cannot resolve " + me.first);
    int lfd = ::socket(sa.ss_family, SOCK_STREAM, 0);
    int one = 1;
    setsockopt(lfd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    if (::bind(lfd, reinterpret_cast<sockaddr*>(&sa), salen) != 0 ||
        ::listen(lfd, world_ * n_channels_ + 8) != 0) {
      std::string err = std::strerror(errno);
      ::close(lfd);
      throw TransportRendezvous("rank " + std::to_string(rank_) + ": cannot listen on " + me.first +
                                ":" + std::to_string(me.second) + ": " + err);
    }
    const int expected_in = (world_ - 1 - rank_) * n_channels_;
    std::atomic<bool> stop{false};
    std::mutex mu;
    std::thread acceptor([&] {
      int accepted = 0;
      while (accepted < expected_in && !stop.load()) {
        pollfd p{lfd, POLLIN, 0};
        int rc = poll(&p, 1, kAcceptPollMs);
        if (rc <= 0) continue;
        int fd = ::accept(lfd, nullptr, nullptr);
        if (fd < 0) continue;
        uint32_t hello[3];
        if (!io_all(fd, reinterpret_cast<char*>(hello), sizeof(hello), false, 10.0) ||
            ntohl(hello[0]) != kHelloMagic) {
          ::close(fd);
          continue;
        }
        int peer = static_cast<int>(ntohl(hello[1]));
        int ch = static_cast<int>(ntohl(hello[2]));
        if (peer <= rank_ || peer >= world_ || ch < 0 || ch >= n_channels_) {
          ::close(fd);
          continue;
        }
        tune_socket(fd);
        std::lock_guard<std::mutex> g(mu);
        int& slot = fds_[static_cast<size_t>(peer) * n_channels_ + ch];
        if (slot >= 0) ::close(slot);
        else accepted++;
        slot = fd;
      }
    });

    std::string failure;
    auto t0 = Clock::now();
    for (int peer = 0; peer < rank_ && failure.empty(); ++peer) {
      sockaddr_storage pa{};
      socklen_t palen = 0;
      if (!resolve(addrs[peer].first, addrs[peer].second, &pa, &palen)) {
        failure = "cannot resolve rank " + std::to_string(peer) + " at " + addrs[peer].first;
        break;
      }
      for (int ch = 0; ch < n_channels_ && failure.empty(); ++ch) {
        int fd = -1;
        while (true) {
          fd = ::socket(pa.ss_family, SOCK_STREAM, 0);
          if (::connect(fd, reinterpret_cast<sockaddr*>(&pa), palen) == 0) break;
          ::close(fd);
          fd = -1;
          if (seconds_since(t0) > timeout_s) break;
          std::this_thread::sleep_for(std::chrono::milliseconds(50));
        }
        if (fd < 0) {
          failure = "could not reach rank " + std::to_string(peer) + " at " + addrs[peer].first + ":" +
                    std::to_string(addrs[peer].second);
          break;
        }
        uint32_t hello[3] = {htonl(kHelloMagic), htonl(static_cast<uint32_t>(rank_)),
                             htonl(static_cast<uint32_t>(ch))};
        if (!io_all(fd, reinterpret_cast<char*>(hello), sizeof(hello), true, 10.0)) {
          ::close(fd);
          failure = "handshake with rank " + std::to_string(peer) + " failed";
          break;
        }
        tune_socket(fd);
        std::lock_guard<std::mutex> g(mu);
        fds_[static_cast<size_t>(peer) * n_channels_ + ch] = fd;
      }
    }
    // Wait for the higher ranks to dial in, within what is left of the budget.
    while (failure.empty()) {
      {
        std::lock_guard<std::mutex> g(mu);
        int have = 0;
        for (int p = rank_ + 1; p < world_; ++p)
          for (int ch = 0; ch < n_channels_; ++ch) have += fds_[static_cast<size_t>(p) * n_channels_ + ch] >= 0;
        if (have == expected_in) break;
      }
      if (seconds_since(t0) > timeout_s) {
        failure = "timed out waiting for higher ranks to connect";
        break;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(20));
    }
    stop.store(true);
    acceptor.join();
    ::close(lfd);
    if (!failure.empty()) {
      std::set<int> missing;
      for (int p = 0; p < world_; ++p) {
        if (p == rank_) continue;
        for (int ch = 0; ch < n_channels_; ++ch)
          if (fds_[static_cast<size_t>(p) * n_channels_ + ch] < 0) missing.insert(p);
      }
      int have = 0;
      for (int fd : fds_) have += fd >= 0;
      close();
      std::ostringstream os;
      os << "rank " << rank_ << ": established " << have << "/" << (world_ - 1) * n_channels_
         << " connections; no contact with ranks [";
      bool first = true;
      for (int p : missing) {
        os << (first ? "" : ", ") << p;
        first = false;
      }
      os << "] (" << failure << ")";
      throw TransportRendezvous(os.str());
    }
    for (int fd : fds_)
      if (fd >= 0) set_nonblocking(fd, true);
  }

  int rank_, world_, n_channels_;
  std::atomic<double> op_timeout_;
  std::vector<int> fds_;
  std::mutex close_mu_;
};

}  // namespace mnb

PYBIND11_MODULE(_host, m) {
  m.doc() = "mini_nccl_b200 native host transport (TCP full mesh)";
  py::register_exception<mnb::TransportTimeout>(m, "TransportTimeout", PyExc_TimeoutError);
  py::register_exception<mnb::TransportPeerClosed>(m, "TransportPeerClosed", PyExc_ConnectionError);
  py::register_exception<mnb::TransportRendezvous>(m, "TransportRendezvous", PyExc_TimeoutError);
  py::class_<mnb::TcpMesh>(m, "TcpMesh")
      .def(py::init<int, int, std::vector<std::pair<std::string, int>>, int, double, double>(),
           py::arg("rank"), py::arg("world_size"), py::arg("addrs"), py::arg("n_channels"),
           py::arg("timeout"), py::arg("op_timeout"))
      .def_property_readonly("rank", &mnb::TcpMesh::rank)
      .def_property_readonly("world_size", &mnb::TcpMesh::world_size)
      .def_property_readonly("n_channels", &mnb::TcpMesh::n_channels)
      .def("set_op_timeout", &mnb::TcpMesh::set_op_timeout)
      .def("op_timeout", &mnb::TcpMesh::op_timeout)
      .def("send", &mnb::TcpMesh::send)
      .def("recv", &mnb::TcpMesh::recv)
      .def("exchange", &mnb::TcpMesh::exchange)
      .def("close", &mnb::TcpMesh::close);
}
