#include "work_output.h"

#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

namespace spc {
namespace wo {

WorkOutput::WorkOutput(const wc::Config& cfg, bool has_next, std::string host, uint32_t port, uint32_t rows,
                       uint32_t queue_capacity, uint32_t release_capacity)
    : cfg_(cfg),
      has_next_(has_next),
      host_(std::move(host)),
      port_(port),
      rows_(rows),
      queue_capacity_(queue_capacity),
      release_capacity_(release_capacity) {
  cfg_.validate();
  if (!queue_capacity || !release_capacity || !rows) fail(Status::InvalidArgument, "work output: zero capacity");
  if (has_next && (host_.empty() || !port || port > 65535)) fail(Status::InvalidArgument, "work output: next rank address");
  ack_.resize(rd::kAckBytes);
}

WorkOutput::~WorkOutput() { drop_socket(); }

void WorkOutput::enqueue(const wc::Packet& p) {
  if (queue_.size() >= queue_capacity_) fail(Status::CapacityExceeded, "work output: queue full");
  wc::validate_packet(p, cfg_);
  if (p.execution_row_count > rows_) fail(Status::InvalidArgument, "work output: packet exceeds the execution rows");
  Item it{p, wc::serialize(p), 0};
  it.fingerprint = wc::fingerprint_bytes(it.bytes.data(), it.bytes.size());
  queue_.push_back(std::move(it));
  ++st_.enqueued;
}

void WorkOutput::adopt_socket(int fd) {
  drop_socket();
  const int fl = fcntl(fd, F_GETFL, 0);
  if (fl < 0 || fcntl(fd, F_SETFL, fl | O_NONBLOCK) < 0) fail(Status::IoError, "work output: socket flags");
  fd_ = fd;
  connecting_ = false;
}

void WorkOutput::drop_socket() {
  if (fd_ >= 0) {
    ::close(fd_);
    ++st_.socket_drops;
  }
  fd_ = -1;
  connecting_ = false;
  write_off_ = 0;  // the head packet goes again, whole, on the next connection
  reset_ack();
}

void WorkOutput::reset_ack() {
  awaiting_ack_ = false;
  ack_off_ = 0;
}

Status WorkOutput::ensure_socket() {
  if (fd_ >= 0 && !connecting_) return Status::Ok;
  if (fd_ < 0) {
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    hints.ai_socktype = SOCK_STREAM;
    if (getaddrinfo(host_.c_str(), std::to_string(port_).c_str(), &hints, &res) != 0 || !res)
      return Status::RouteNotFound;
    const int fd = ::socket(res->ai_family, res->ai_socktype | SOCK_NONBLOCK, 0);
    if (fd < 0) {
      freeaddrinfo(res);
      return Status::RouteNotFound;
    }
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
    const int rc = ::connect(fd, res->ai_addr, res->ai_addrlen);
    freeaddrinfo(res);
    if (rc != 0 && errno != EINPROGRESS) {
      ::close(fd);
      return Status::RouteNotFound;
    }
    fd_ = fd;
    connecting_ = rc != 0;
    if (!connecting_) return Status::Ok;
  }
  // a non-blocking connect in progress: writable once it completes
  int err = 0;
  socklen_t len = sizeof err;
  char probe;
  if (getsockopt(fd_, SOL_SOCKET, SO_ERROR, &err, &len) != 0 || err != 0) {
    drop_socket();
    return Status::RouteNotFound;
  }
  const ssize_t r = ::recv(fd_, &probe, 0, MSG_DONTWAIT);
  (void)r;
  sockaddr_storage peer;
  socklen_t plen = sizeof peer;
  if (getpeername(fd_, reinterpret_cast<sockaddr*>(&peer), &plen) != 0) return Status::Busy;  // not connected yet
  connecting_ = false;
  return Status::Ok;
}

Status WorkOutput::pump(const FailFn& on_hard_failure) {
  if (!has_next_ || queue_.empty()) return Status::Ok;
  const Status s = ensure_socket();
  if (s != Status::Ok) return s;
  while (!queue_.empty()) {
    Item& head = queue_.front();
    if (!awaiting_ack_) {
      while (write_off_ < head.bytes.size()) {
        const ssize_t n = ::send(fd_, head.bytes.data() + write_off_, head.bytes.size() - write_off_,
                                 MSG_NOSIGNAL | MSG_DONTWAIT);
        if (n > 0) {
          write_off_ += size_t(n);
          continue;
        }
        if (n < 0 && errno == EINTR) continue;
        if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) return Status::Busy;
        drop_socket();
        return Status::RouteNotFound;
      }
      ++st_.sent;
      if (resending_) ++st_.resent;
      awaiting_ack_ = true;
      ack_off_ = 0;
    }
    while (ack_off_ < rd::kAckBytes) {
      const ssize_t n = ::recv(fd_, &ack_[ack_off_], rd::kAckBytes - ack_off_, MSG_DONTWAIT);
      if (n > 0) {
        ack_off_ += size_t(n);
        continue;
      }
      if (n < 0 && errno == EINTR) continue;
      if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) return Status::Busy;
      drop_socket();  // closed (n == 0) or failed
      return Status::RouteNotFound;
    }
    rd::Ack a;
    try {
      a = rd::ack_from_wire(ack_);
    } catch (const StatusError&) {
      drop_socket();  // the stream is out of step: start over on a new connection
      return Status::RouteNotFound;
    }
    const std::string want = rd::identity_to_wire(head.packet.identity);
    if (rd::identity_to_wire(a.identity) != want || a.packet_fingerprint != head.fingerprint) {
      drop_socket();
      return Status::RouteNotFound;
    }
    reset_ack();
    write_off_ = 0;
    const Status as = Status(a.status);
    if (as == Status::CapacityExceeded) {  // the next rank's queue was full: resend later
      resending_ = true;
      return Status::Busy;
    }
    resending_ = false;
    if (as == Status::Ok) {
      ++st_.acknowledged;
    } else if (as == Status::Duplicate) {
      ++st_.duplicates;
    } else {
      ++st_.hard_failures;
      if (on_hard_failure) on_hard_failure(head.packet, as);
    }
    queue_.pop_front();
  }
  return Status::Ok;
}

void WorkOutput::queue_release(const ReleaseRecord& r) {
  if (releases_.size() >= release_capacity_) fail(Status::CapacityExceeded, "work output: release ring full");
  if (!r.request_id || !r.sequence_id || !r.token_count)
    fail(Status::InvalidArgument, "work output: release record needs ids and a token count");
  releases_.push_back(r);
  ++st_.releases_queued;
}

wc::Packet WorkOutput::build_release_packet(const wc::Identity& id, uint32_t lanes) const {
  if (releases_.empty() || !lanes) fail(Status::InvalidArgument, "work output: nothing to release");
  wc::Packet p;
  p.flags = wc::kFlagReleaseSequences;
  p.identity = id;
  p.identity.transaction_phase = wc::kPhaseRelease;
  const uint32_t n = std::min<uint32_t>(lanes, uint32_t(releases_.size()));
  for (uint32_t i = 0; i < n; ++i) {
    const ReleaseRecord& r = releases_[i];
    wc::Lane l;
    l.request_id = r.request_id;
    l.request_generation = r.request_generation;
    l.step_generation = id.step_generation;
    l.sequence_id = r.sequence_id;
    l.context_token_count = r.token_count;
    l.request_slot_index = i;
    p.lanes.push_back(l);
  }
  p.request_id = releases_[0].request_id;
  p.sequence_id = releases_[0].sequence_id;
  p.active_sequence_count = n;
  p.execution_row_count = n;
  p.block_token_count = cfg_.kv_block_tokens;
  p.max_blocks_per_sequence = cfg_.kv_block_capacity();
  return p;
}

void WorkOutput::pop_releases(uint32_t n) {
  if (n > releases_.size()) fail(Status::InvalidArgument, "work output: popping more releases than queued");
  releases_.erase(releases_.begin(), releases_.begin() + n);
  st_.releases_sent += n;
}

}  // namespace wo
}  // namespace spc
