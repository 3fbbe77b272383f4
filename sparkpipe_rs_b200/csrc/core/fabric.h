// Multi-node host fabric: the neighbour transfer plane (memlink) and the fabric
// topology model of a ring of nodes.
//
// memlink   a buffer moves to a ring neighbour over `lanes` parallel TCP
//           connections (ports base_port + lane), each lane carrying one
//           contiguous, chunk-aligned share of the bytes in 1 MiB writes.
//           Planning helpers (lane partition, neighbour rank, host-name template,
//           neighbour endpoint) are pure functions; `Memlink::send` / `receive` do
//           the transfer with one thread per lane.
// topology  the three fabric layouts of a node ring: a debug ring with one rail
//           (each node cabled to its two neighbours), one switch with one rail,
//           and a two-switch two-rail layout (described and validated, not yet
//           routable). Validation checks the layout's rail / switch / port counts,
//           100 Gb/s links and a 1500-9600 byte MTU; route resolution returns the
//           first hop, the port, the rail and the hop count to a destination node.
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_memlink.h:13-69
// (defaults: base port 55200, 8 lanes, at most 64, 1 GiB store, 1 MiB chunks; the
// planning calls) and spark_fabric_topology.h:12-80 (modes, flags, link speed, MTU
// bounds, route record). The reference declares these without an implementation;
// the rules here are this framework's own.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace fabric {

constexpr uint16_t kDefaultBasePort = 55200;
constexpr uint32_t kDefaultLanes = 8;
constexpr uint32_t kMaxLanes = 64;
constexpr uint32_t kMaxHostBytes = 255;
constexpr uint64_t kDefaultStoreBytes = 1ull << 30;
constexpr uint64_t kChunkBytes = 1ull << 20;

struct Partition {
  uint32_t lane = 0, lanes = 0;
  uint64_t offset = 0, bytes = 0;
};

struct Endpoint {
  std::string host;
  uint16_t base_port = kDefaultBasePort;
  uint32_t lanes = kDefaultLanes;
};

enum class Direction : uint32_t { Previous = 0, Next = 1 };

void validate_lanes(uint32_t lanes);
// Lane `lane` of `lanes` gets chunks [floor(lane * C / lanes), floor((lane + 1) * C / lanes))
// of the C = ceil(total / chunk) chunks, clipped to `total`.
Partition partition(uint64_t total, uint32_t lanes, uint32_t lane, uint64_t chunk = kChunkBytes);
uint32_t neighbor_rank(uint32_t rank, uint32_t ranks, Direction d);
// Replaces every "{rank}" in the template with the rank's decimal value.
std::string host_from_template(const std::string& tmpl, uint32_t rank);
Endpoint neighbor_endpoint(uint32_t rank, uint32_t ranks, Direction d, const std::string& host_template,
                           uint16_t base_port = kDefaultBasePort, uint32_t lanes = kDefaultLanes);

// Multi-lane TCP transfer of one buffer. receive() listens on base_port + lane for
// every lane, accepts one connection per lane and fills `dst` (which must hold the
// sender's total); send() connects every lane and writes its partition. Each lane
// first sends a 40-byte header (magic, total, lane, lanes, offset, bytes) that the
// receiver checks against its own partition. Both return the bytes moved; a
// timeout or a mismatch raises.
class Memlink {
 public:
  static uint64_t send(const std::string& host, uint16_t base_port, uint32_t lanes, const uint8_t* src,
                       uint64_t total, uint32_t timeout_ms = 30000);
  static uint64_t receive(uint16_t base_port, uint32_t lanes, uint8_t* dst, uint64_t capacity,
                          uint32_t timeout_ms = 30000);
};

enum class Mode : uint32_t { Invalid = 0, RingDebugSingleRail = 1, SingleSwitchSingleRail = 2, DualSwitchDualRail = 3 };
constexpr uint32_t kFlagDebugOnly = 0x1;
constexpr uint32_t kFlagSwitched = 0x2;
constexpr uint32_t kFlagFutureOnly = 0x4;
constexpr uint32_t kLinkGbps = 100;
constexpr uint32_t kMinMtu = 1500;
constexpr uint32_t kMaxMtu = 9600;
constexpr uint32_t kNoNode = 0xffffffffu;
constexpr uint32_t kMaxNodes = 1024;

struct TopologyConfig {
  Mode mode = Mode::Invalid;
  uint32_t flags = 0;
  uint32_t nodes = 0;
  uint32_t local = 0;
  uint32_t rails = 0;
  uint32_t switches = 0;
  uint32_t ports = 0;
  uint32_t link_gbps = kLinkGbps;
  uint32_t mtu = kMinMtu;
};

struct Route {
  Mode mode = Mode::Invalid;
  uint32_t rail = 0;
  uint32_t src = 0, dst = 0;
  uint32_t port = 0;
  uint32_t first_hop = kNoNode;  // the next node, or kNoNode through a switch
  uint32_t hops = 0;             // links traversed
  bool switched = false;
};

// A standard configuration of a mode for `nodes` nodes (the fields validate() wants).
TopologyConfig default_topology(Mode mode, uint32_t nodes, uint32_t local, uint32_t mtu = 9000);
void validate(const TopologyConfig& c);
Route resolve_route(const TopologyConfig& c, uint32_t dst);
const char* mode_name(Mode m);

}  // namespace fabric
}  // namespace spc
