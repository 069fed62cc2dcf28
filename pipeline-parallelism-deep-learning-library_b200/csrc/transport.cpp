// transport.cpp -- byte transports between pipeline ranks on the host (crates/transport rebuilt).
//
// The pipeline's own data plane is NCCL over NVLink; these transports carry the reference's
// framed messages where the ranks are host processes or threads (CPU ranks, interop with the
// reference's own ranks, tests of the wire format):
//   loopback        ranks of one process, one FIFO per (destination, source) pair
//                   (crates/transport/src/loopback.rs:21-76);
//   localhost mesh  ranks of one process over 127.0.0.1 sockets (crates/transport/src/tcp.rs:208-231);
//   tcp mesh        one rank per process: rank r listens on addrs[r], dials every lower rank in
//                   order and accepts every higher one, each connection opening with the
//                   12-byte hello "LNGM", world, rank (crates/transport/src/mesh.rs:1-120).
// On a socket every message is a frame: little-endian u64 payload length, then the payload
// (crates/transport/src/tcp.rs:1-3).  Per peer a writer thread drains a bounded outbox (send
// copies once and returns, and blocks while `depth` messages are queued) and a reader thread
// reads frames ahead into an unbounded inbox.  A write error, end of stream or a read error fails
// the outbox (later sends fail) and closes the inbox (queued messages are still delivered, then
// receives fail).  Every failure is LC_ERR_TRANSPORT (the reference's Error::Transport).
#include <arpa/inet.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/uio.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

using Clock = std::chrono::steady_clock;

namespace {

using lc::fail;

constexpr uint32_t kDefaultDepth = 4;       // messages a sender may queue per peer (tcp.rs:21)
constexpr uint64_t kGrowStep = 1ull << 20;  // reader allocates at most this far ahead of the data
constexpr int kRetryMs = 5;                 // pause between dial / accept attempts (mesh.rs:22)
constexpr int kReaderGraceMs = 1000;        // how long destroy waits for a reader (tcp.rs:28)
constexpr uint32_t kHelloLen = 12;

using Message = std::vector<uint8_t>;

// Deadline from a timeout in ms; a negative timeout never expires.
struct Deadline {
  bool forever;
  Clock::time_point at;
  explicit Deadline(int64_t ms) : forever(ms < 0), at(Clock::now() + std::chrono::milliseconds(ms < 0 ? 0 : ms)) {}
  bool passed() const { return !forever && Clock::now() >= at; }
  int64_t left_ms() const {
    if (forever) return -1;
    auto d = std::chrono::duration_cast<std::chrono::milliseconds>(at - Clock::now()).count();
    return d > 0 ? d : 0;
  }
};

// FIFO of messages with a timed pop.  Once closed, pops deliver what is queued, then fail.
struct Inbox {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<Message> q;
  bool closed = false;

  void push(Message&& m) {
    {
      std::lock_guard<std::mutex> g(mu);
      q.push_back(std::move(m));
    }
    cv.notify_one();
  }
  void close() {
    {
      std::lock_guard<std::mutex> g(mu);
      closed = true;
    }
    cv.notify_all();
  }
  bool wait_closed(int64_t ms) {
    std::unique_lock<std::mutex> lk(mu);
    return cv.wait_for(lk, std::chrono::milliseconds(ms), [&] { return closed; });
  }
  lc_status pop(Message* out, int64_t timeout_ms) {
    const Deadline dl(timeout_ms);
    std::unique_lock<std::mutex> lk(mu);
    for (;;) {
      if (!q.empty()) {
        *out = std::move(q.front());
        q.pop_front();
        return LC_OK;
      }
      if (closed) return fail(LC_ERR_TRANSPORT, "the peer is gone");
      if (dl.forever) {
        cv.wait(lk);
      } else {
        if (dl.passed()) return fail(LC_ERR_TRANSPORT, "receive timed out");
        cv.wait_until(lk, dl.at);
      }
    }
  }
};

// Bounded queue from `send` to a peer's writer thread.
struct Outbox {
  std::mutex mu;
  std::condition_variable not_full, not_empty;
  std::deque<Message> q;
  size_t depth;
  size_t slots = 0;   // queued messages plus senders filling a buffer
  bool failed = false;  // the connection is unusable
  bool closed = false;  // the endpoint is going away: drain, then stop
  explicit Outbox(size_t d) : depth(d) {}

  lc_status push_parts(const void* const* parts, const uint64_t* lens, uint32_t n) {
    uint64_t total = 0;
    for (uint32_t i = 0; i < n; i++)
      if (__builtin_add_overflow(total, lens[i], &total)) return fail(LC_ERR_TRANSPORT, "message length overflows");
    {
      std::unique_lock<std::mutex> lk(mu);
      not_full.wait(lk, [&] { return failed || slots < depth; });
      if (failed) return fail(LC_ERR_TRANSPORT, "the connection to the peer failed");
      slots++;
    }
    Message m;
    m.reserve(total);
    for (uint32_t i = 0; i < n; i++) {
      const uint8_t* p = static_cast<const uint8_t*>(parts[i]);
      m.insert(m.end(), p, p + lens[i]);
    }
    {
      std::lock_guard<std::mutex> g(mu);
      if (failed) {
        slots--;
        not_full.notify_one();
        return fail(LC_ERR_TRANSPORT, "the connection to the peer failed");
      }
      q.push_back(std::move(m));
    }
    not_empty.notify_one();
    return LC_OK;
  }
  // The writer's next message; false once failed, or closed and drained.
  bool pop(Message* out) {
    std::unique_lock<std::mutex> lk(mu);
    not_empty.wait(lk, [&] { return failed || closed || !q.empty(); });
    if (failed || q.empty()) return false;
    *out = std::move(q.front());
    q.pop_front();
    return true;
  }
  void done_one() {
    {
      std::lock_guard<std::mutex> g(mu);
      slots--;
    }
    not_full.notify_one();
  }
  void fail_now() {
    {
      std::lock_guard<std::mutex> g(mu);
      failed = true;
    }
    not_full.notify_all();
    not_empty.notify_all();
  }
  void close() {
    {
      std::lock_guard<std::mutex> g(mu);
      closed = true;
    }
    not_empty.notify_all();
  }
};

// ---- sockets --------------------------------------------------------------------------------

bool write_all(int fd, const void* p, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(p);
  while (n > 0) {
    const ssize_t w = ::send(fd, b, n, MSG_NOSIGNAL);
    if (w < 0 && errno == EINTR) continue;
    if (w <= 0) return false;
    b += w;
    n -= (size_t)w;
  }
  return true;
}

bool read_all(int fd, void* p, size_t n) {
  uint8_t* b = static_cast<uint8_t*>(p);
  while (n > 0) {
    const ssize_t r = ::recv(fd, b, n, 0);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    b += r;
    n -= (size_t)r;
  }
  return true;
}

// One frame: the u64 little-endian length and the payload, gathered into as few writes as the
// socket takes.
bool write_frame(int fd, const Message& m) {
  uint8_t hdr[8];
  const uint64_t len = m.size();
  for (int i = 0; i < 8; i++) hdr[i] = (uint8_t)(len >> (8 * i));
  iovec iov[2] = {{hdr, 8}, {const_cast<uint8_t*>(m.data()), m.size()}};
  size_t left = 8 + m.size();
  int first = 0;
  while (left > 0) {
    msghdr mh{};
    mh.msg_iov = iov + first;
    mh.msg_iovlen = 2 - first;
    const ssize_t w = ::sendmsg(fd, &mh, MSG_NOSIGNAL);
    if (w < 0 && errno == EINTR) continue;
    if (w <= 0) return false;
    size_t done = (size_t)w;
    left -= done;
    while (done > 0 && first < 2) {
      if (done >= iov[first].iov_len) {
        done -= iov[first].iov_len;
        iov[first].iov_len = 0;
        first++;
      } else {
        iov[first].iov_base = static_cast<uint8_t*>(iov[first].iov_base) + done;
        iov[first].iov_len -= done;
        done = 0;
      }
    }
  }
  return true;
}

// Reads a payload of `len` bytes, growing the buffer only as data arrives, so a corrupt length
// cannot make the reader allocate more than the peer actually sends.
bool read_payload(int fd, Message* m, uint64_t len) {
  m->clear();
  uint64_t filled = 0;
  while (filled < len) {
    const uint64_t step = std::min<uint64_t>(len - filled, std::max<uint64_t>(filled, kGrowStep));
    m->resize(filled + step);
    if (!read_all(fd, m->data() + filled, step)) return false;
    filled += step;
  }
  return true;
}

void tune(int fd) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  int buf = 4 << 20;  // large socket buffers: 4 MiB messages stream without stalls
  setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &buf, sizeof(buf));
  setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &buf, sizeof(buf));
}

void set_io_timeout(int fd, int64_t ms) {
  timeval tv{};
  if (ms > 0) {
    tv.tv_sec = ms / 1000;
    tv.tv_usec = (ms % 1000) * 1000;
  }
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
  setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
}

// One connection: its socket, queues and the two threads that move frames.  Shared with the
// threads, so a reader that outlives the endpoint (it is detached after the grace period) still
// owns what it touches.
struct Peer {
  int fd = -1;
  Outbox out;
  Inbox in;
  std::thread writer, reader;
  Peer(int f, size_t depth) : fd(f), out(depth) {}
  ~Peer() {
    if (fd >= 0) ::close(fd);
  }
};

void start_peer(const std::shared_ptr<Peer>& p) {
  tune(p->fd);
  std::shared_ptr<Peer> w = p, r = p;
  p->writer = std::thread([w] {
    Message m;
    while (w->out.pop(&m)) {
      const bool ok = write_frame(w->fd, m);
      w->out.done_one();
      if (!ok) {
        w->out.fail_now();
        ::shutdown(w->fd, SHUT_RDWR);  // wakes the reader, which closes the inbox
        return;
      }
    }
  });
  p->reader = std::thread([r] {
    for (;;) {
      uint8_t hdr[8];
      if (!read_all(r->fd, hdr, 8)) break;
      uint64_t len = 0;
      for (int i = 0; i < 8; i++) len |= (uint64_t)hdr[i] << (8 * i);
      Message m;
      if (!read_payload(r->fd, &m, len)) break;
      r->in.push(std::move(m));
    }
    r->out.fail_now();  // the peer is gone: later sends fail instead of queueing
    ::shutdown(r->fd, SHUT_RDWR);
    r->in.close();
  });
}

void stop_peer(const std::shared_ptr<Peer>& p) {
  p->out.close();  // queued messages go out first
  if (p->writer.joinable()) p->writer.join();
  ::shutdown(p->fd, SHUT_RDWR);
  if (p->reader.joinable()) {
    if (p->in.wait_closed(kReaderGraceMs)) p->reader.join();
    else p->reader.detach();
  }
}

struct Hub {  // loopback: box[dest * world + src]
  uint32_t world;
  std::vector<Inbox> boxes;
  explicit Hub(uint32_t w) : world(w), boxes((size_t)w * w) {}
};

}  // namespace

struct lc_transport {
  uint32_t rank = 0, world = 0;
  std::shared_ptr<Hub> hub;                    // loopback
  std::vector<std::shared_ptr<Peer>> peers;    // tcp: indexed by rank, null at our own
};

namespace {

lc_status check_rank(const lc_transport* t, uint32_t other) {
  if (t == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null transport");
  if (other >= t->world || other == t->rank) return fail(LC_ERR_TRANSPORT, "peer rank out of range or our own");
  if (!t->hub && !t->peers[other]) return fail(LC_ERR_TRANSPORT, "no connection to that rank");
  return LC_OK;
}

lc_status make_tcp(uint32_t rank, std::vector<int>& fds, uint32_t depth, lc_transport** out) {
  auto* t = new lc_transport();
  t->rank = rank;
  t->world = (uint32_t)fds.size();
  t->peers.resize(fds.size());
  for (size_t r = 0; r < fds.size(); r++) {
    if (fds[r] < 0) continue;
    t->peers[r] = std::make_shared<Peer>(fds[r], depth);
    fds[r] = -1;
    start_peer(t->peers[r]);
  }
  *out = t;
  return LC_OK;
}

bool parse_addr(const char* s, sockaddr_in* a) {
  if (s == nullptr) return false;
  const char* colon = strrchr(s, ':');
  if (colon == nullptr) return false;
  std::string host(s, colon - s);
  if (host == "localhost") host = "127.0.0.1";
  char* end = nullptr;
  const long port = strtol(colon + 1, &end, 10);
  if (end == colon + 1 || *end != 0 || port < 0 || port > 65535) return false;
  memset(a, 0, sizeof(*a));
  a->sin_family = AF_INET;
  a->sin_port = htons((uint16_t)port);
  return inet_pton(AF_INET, host.c_str(), &a->sin_addr) == 1;
}

int listen_on(const sockaddr_in& a) {
  const int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) return -1;
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  if (::bind(fd, reinterpret_cast<const sockaddr*>(&a), sizeof(a)) != 0 || ::listen(fd, 64) != 0) {
    ::close(fd);
    return -1;
  }
  return fd;
}

void hello(uint8_t out[kHelloLen], uint32_t world, uint32_t rank) {
  memcpy(out, "LNGM", 4);
  for (int i = 0; i < 4; i++) out[4 + i] = (uint8_t)(world >> (8 * i));
  for (int i = 0; i < 4; i++) out[8 + i] = (uint8_t)(rank >> (8 * i));
}

bool read_hello(int fd, uint32_t* world, uint32_t* rank) {
  uint8_t b[kHelloLen];
  if (!read_all(fd, b, kHelloLen) || memcmp(b, "LNGM", 4) != 0) return false;
  *world = *rank = 0;
  for (int i = 0; i < 4; i++) *world |= (uint32_t)b[4 + i] << (8 * i);
  for (int i = 0; i < 4; i++) *rank |= (uint32_t)b[8 + i] << (8 * i);
  return true;
}

// Dials `a` until it connects or the deadline passes; a connection to ourselves (TCP
// simultaneous open on a local port nobody listens on yet) is not the peer and is retried.
int dial(const sockaddr_in& a, const Deadline& dl) {
  for (;;) {
    if (dl.passed()) return -1;
    const int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) return -1;
    if (::connect(fd, reinterpret_cast<const sockaddr*>(&a), sizeof(a)) == 0) {
      sockaddr_in l{}, r{};
      socklen_t ll = sizeof(l), rl = sizeof(r);
      const bool self = getsockname(fd, reinterpret_cast<sockaddr*>(&l), &ll) == 0 &&
                        getpeername(fd, reinterpret_cast<sockaddr*>(&r), &rl) == 0 && l.sin_port == r.sin_port &&
                        l.sin_addr.s_addr == r.sin_addr.s_addr;
      if (!self) return fd;
    }
    ::close(fd);
    std::this_thread::sleep_for(std::chrono::milliseconds(kRetryMs));
  }
}

int accept_until(int lfd, const Deadline& dl) {
  for (;;) {
    if (dl.passed()) return -1;
    pollfd p{lfd, POLLIN, 0};
    const int64_t left = dl.left_ms();
    const int wait = left < 0 ? kRetryMs * 20 : (int)std::min<int64_t>(left, kRetryMs * 20);
    const int r = ::poll(&p, 1, wait);
    if (r < 0 && errno != EINTR) return -1;
    if (r <= 0) continue;
    const int fd = ::accept4(lfd, nullptr, nullptr, SOCK_CLOEXEC);
    if (fd >= 0) return fd;
    if (errno != EINTR && errno != EAGAIN && errno != ECONNABORTED) return -1;
  }
}

void close_all(std::vector<int>& fds) {
  for (int& f : fds)
    if (f >= 0) {
      ::close(f);
      f = -1;
    }
}

}  // namespace

extern "C" {

lc_status lc_transport_loopback(uint32_t world, lc_transport** out) {
  if (out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null output");
  if (world < 2) return fail(LC_ERR_TRANSPORT, "a mesh needs at least two ranks");
  auto hub = std::make_shared<Hub>(world);
  for (uint32_t r = 0; r < world; r++) {
    out[r] = new lc_transport();
    out[r]->rank = r;
    out[r]->world = world;
    out[r]->hub = hub;
  }
  return LC_OK;
}

lc_status lc_transport_localhost_mesh(uint32_t world, lc_transport** out) {
  if (out == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null output");
  if (world < 2) return fail(LC_ERR_TRANSPORT, "a mesh needs at least two ranks");
  std::vector<int> listeners(world, -1);
  std::vector<std::vector<int>> fds(world, std::vector<int>(world, -1));
  auto cleanup = [&] {
    close_all(listeners);
    for (auto& row : fds) close_all(row);
  };
  sockaddr_in any{};
  any.sin_family = AF_INET;
  any.sin_addr.s_addr = htonl(INADDR_LOOPBACK);
  std::vector<sockaddr_in> addrs(world);
  for (uint32_t r = 0; r < world; r++) {
    listeners[r] = listen_on(any);
    socklen_t len = sizeof(addrs[r]);
    if (listeners[r] < 0 || getsockname(listeners[r], reinterpret_cast<sockaddr*>(&addrs[r]), &len) != 0) {
      cleanup();
      return fail(LC_ERR_TRANSPORT, "could not listen on 127.0.0.1");
    }
  }
  // each connection completes in the listener's backlog, so connect then accept from one
  // thread cannot deadlock
  for (uint32_t lo = 0; lo < world; lo++)
    for (uint32_t hi = lo + 1; hi < world; hi++) {
      const int d = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
      if (d < 0 || ::connect(d, reinterpret_cast<const sockaddr*>(&addrs[hi]), sizeof(addrs[hi])) != 0) {
        if (d >= 0) ::close(d);
        cleanup();
        return fail(LC_ERR_TRANSPORT, "could not connect over 127.0.0.1");
      }
      const int a = ::accept4(listeners[hi], nullptr, nullptr, SOCK_CLOEXEC);
      if (a < 0) {
        ::close(d);
        cleanup();
        return fail(LC_ERR_TRANSPORT, "could not accept over 127.0.0.1");
      }
      fds[lo][hi] = d;
      fds[hi][lo] = a;
    }
  close_all(listeners);
  for (uint32_t r = 0; r < world; r++) make_tcp(r, fds[r], kDefaultDepth, &out[r]);
  return LC_OK;
}

lc_status lc_transport_tcp_mesh(uint32_t rank, const char* const* addrs, uint32_t world, int64_t connect_timeout_ms,
                                uint32_t queue_depth, lc_transport** out) {
  if (out == nullptr || addrs == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  if (world < 2 || rank >= world || queue_depth == 0)
    return fail(LC_ERR_TRANSPORT, "a mesh needs two or more ranks, a rank below the world and a queue depth");
  std::vector<sockaddr_in> sa(world);
  for (uint32_t r = 0; r < world; r++)
    if (!parse_addr(addrs[r], &sa[r])) return fail(LC_ERR_TRANSPORT, "address is not IPv4 host:port");
  const Deadline dl(connect_timeout_ms);
  std::vector<int> fds(world, -1);
  const int lfd = listen_on(sa[rank]);
  if (lfd < 0) return fail(LC_ERR_TRANSPORT, "could not listen on this rank's address");
  auto bail = [&](const char* why) {
    ::close(lfd);
    close_all(fds);
    return fail(LC_ERR_TRANSPORT, why);
  };
  uint8_t mine[kHelloLen];
  hello(mine, world, rank);
  // every lower rank, in order: dial, send our hello, check theirs
  for (uint32_t lower = 0; lower < rank; lower++) {
    const int fd = dial(sa[lower], dl);
    if (fd < 0) return bail("a lower rank did not answer before the connect timeout");
    set_io_timeout(fd, dl.forever ? 0 : std::max<int64_t>(1, dl.left_ms()));
    uint32_t w = 0, r = 0;
    const bool ok = write_all(fd, mine, kHelloLen) && read_hello(fd, &w, &r) && w == world && r == lower;
    fds[lower] = fd;
    if (!ok) return bail("handshake with a lower rank failed");
  }
  // every higher rank, in any order: check its hello, answer with ours
  for (uint32_t n = rank + 1; n < world; n++) {
    const int fd = accept_until(lfd, dl);
    if (fd < 0) return bail("a higher rank did not connect before the connect timeout");
    set_io_timeout(fd, dl.forever ? 0 : std::max<int64_t>(1, dl.left_ms()));
    uint32_t w = 0, r = 0;
    if (!read_hello(fd, &w, &r) || w != world || r <= rank || r >= world || fds[r] >= 0) {
      ::close(fd);
      return bail("handshake with a higher rank failed");
    }
    fds[r] = fd;
    if (!write_all(fd, mine, kHelloLen)) return bail("handshake with a higher rank failed");
  }
  ::close(lfd);
  for (int fd : fds)
    if (fd >= 0) set_io_timeout(fd, 0);
  return make_tcp(rank, fds, queue_depth, out);
}

lc_status lc_transport_destroy(lc_transport* t) {
  if (t == nullptr) return LC_OK;
  for (auto& p : t->peers)
    if (p) stop_peer(p);
  delete t;
  return LC_OK;
}

uint32_t lc_transport_rank(const lc_transport* t) { return t ? t->rank : 0; }
uint32_t lc_transport_world(const lc_transport* t) { return t ? t->world : 0; }

lc_status lc_transport_send_parts(lc_transport* t, uint32_t dest, const void* const* parts, const uint64_t* lens,
                                  uint32_t n_parts) {
  lc_status st = check_rank(t, dest);
  if (st) return st;
  if (n_parts > 0 && (parts == nullptr || lens == nullptr)) return fail(LC_ERR_INVALID_ARGUMENT, "null parts");
  for (uint32_t i = 0; i < n_parts; i++)
    if (parts[i] == nullptr && lens[i] > 0) return fail(LC_ERR_INVALID_ARGUMENT, "null part");
  if (t->hub) {
    uint64_t total = 0;
    for (uint32_t i = 0; i < n_parts; i++)
      if (__builtin_add_overflow(total, lens[i], &total)) return fail(LC_ERR_TRANSPORT, "message length overflows");
    Message m;
    m.reserve(total);
    for (uint32_t i = 0; i < n_parts; i++) {
      const uint8_t* p = static_cast<const uint8_t*>(parts[i]);
      m.insert(m.end(), p, p + lens[i]);
    }
    t->hub->boxes[(size_t)dest * t->world + t->rank].push(std::move(m));
    return LC_OK;
  }
  return t->peers[dest]->out.push_parts(parts, lens, n_parts);
}

lc_status lc_transport_send(lc_transport* t, uint32_t dest, const void* bytes, uint64_t len) {
  const void* parts[1] = {bytes};
  return lc_transport_send_parts(t, dest, parts, &len, 1);
}

lc_status lc_transport_recv(lc_transport* t, uint32_t src, int64_t timeout_ms, uint8_t** data, uint64_t* len) {
  lc_status st = check_rank(t, src);
  if (st) return st;
  if (data == nullptr || len == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null output");
  Message m;
  st = t->hub ? t->hub->boxes[(size_t)t->rank * t->world + src].pop(&m, timeout_ms)
              : t->peers[src]->in.pop(&m, timeout_ms);
  if (st) return st;
  uint8_t* buf = static_cast<uint8_t*>(malloc(m.empty() ? 1 : m.size()));
  if (buf == nullptr) return fail(LC_ERR_TRANSPORT, "out of host memory");
  if (!m.empty()) memcpy(buf, m.data(), m.size());
  *data = buf;
  *len = m.size();
  return LC_OK;
}

void lc_transport_free(uint8_t* data) { free(data); }

}  // extern "C"

// ---- framed device tensors: the pipeline's send_tensor / recv_tensor -------------------------
// crates/pipeline/src/lib.rs:71-98: download the tensor, frame it with the LNGL header
// (crates/core/src/lib.rs:298-412) and send it; receive, check the dtype and shape, upload.

extern "C" {

lc_status lc_transport_send_tensor(lc_transport* t, uint32_t dest, lc_context* ctx, const lc_view* v) {
  if (ctx == nullptr || v == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  lc_status st = check_rank(t, dest);
  if (!st) st = lc::validate(*v, "tensor");
  if (st) return st;
  if (!lc::packed_layout(*v)) return fail(LC_ERR_SHAPE, "a framed tensor is row-major contiguous at offset 0");
  uint8_t header[48];
  uint64_t hlen = 0;
  if ((st = lc_wire_write_header(v->dtype, v->shape, (uint32_t)v->rank, header, &hlen))) return st;
  const uint64_t bytes = lc::numel(*v) * lc::dtype_size(v->dtype);
  std::vector<uint8_t> payload(bytes);
  if (bytes > 0) {
    cudaError_t e = cudaMemcpyAsync(payload.data(), v->data, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return lc::cuda_fail(e, "download of a framed tensor");
  }
  const void* parts[2] = {header, payload.data()};
  const uint64_t lens[2] = {hlen, bytes};
  return lc_transport_send_parts(t, dest, parts, lens, 2);
}

lc_status lc_transport_recv_tensor(lc_transport* t, uint32_t src, int64_t timeout_ms, lc_context* ctx,
                                   const lc_view* v) {
  if (ctx == nullptr || v == nullptr) return fail(LC_ERR_INVALID_ARGUMENT, "null argument");
  lc_status st = check_rank(t, src);
  if (!st) st = lc::validate(*v, "tensor");
  if (st) return st;
  if (!lc::packed_layout(*v)) return fail(LC_ERR_SHAPE, "a framed tensor is row-major contiguous at offset 0");
  uint8_t* msg = nullptr;
  uint64_t len = 0;
  if ((st = lc_transport_recv(t, src, timeout_ms, &msg, &len))) return st;
  std::unique_ptr<uint8_t, void (*)(uint8_t*)> hold(msg, lc_transport_free);
  lc_dtype dt = 0;
  uint64_t shape[8] = {};
  uint32_t nd = 0;
  uint64_t off = 0;
  if ((st = lc_wire_parse_header(msg, len, &dt, shape, &nd, &off))) return st;
  if (dt != v->dtype) return fail(LC_ERR_DTYPE, "the received tensor has another element type");
  if ((int32_t)nd != v->rank || memcmp(shape, v->shape, sizeof(uint64_t) * nd) != 0)
    return fail(LC_ERR_SHAPE, "the received tensor has another shape");
  const uint64_t bytes = len - off;
  if (bytes > 0) {
    cudaError_t e = cudaMemcpyAsync(v->data, msg + off, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return lc::cuda_fail(e, "upload of a framed tensor");
  }
  return LC_OK;
}

}  // extern "C"
