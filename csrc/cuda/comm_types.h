// Host- and device-visible types shared by the runtime and the kernels.
//
// Element codes follow the reference wire format (nexar/src/types.rs:13-24,
// `DataType` repr(u8) 0..9); FP8 E4M3 = 10 and E5M2 = 11 are additions for the
// block-scaled fp8 paths and do not renumber the reference codes.
#pragma once
#include <cstddef>

namespace nexar {

enum DType : int {
  kF32 = 0, kF64 = 1, kF16 = 2, kBF16 = 3, kI8 = 4, kI32 = 5, kI64 = 6,
  kU8 = 7, kU32 = 8, kU64 = 9, kF8E4M3 = 10, kF8E5M2 = 11,
};

// Reduce operator codes follow nexar/src/types.rs:62-71 (Sum, Prod, Min, Max).
enum RedOp : int { kSum = 0, kProd = 1, kMin = 2, kMax = 3 };

// Device status word layout (host-mapped; written with plain stores and a
// system-scope fence, the code field last).
// A kernel that gives up waiting on a peer writes these and returns normally,
// so the context stays usable and the host can map the code to an error.
struct DeviceStatus {
  unsigned int code;      // 0 = ok, otherwise a StatusCode below
  unsigned int rank;      // rank whose flag never arrived
  unsigned int op;        // collective op id
  unsigned int block;     // block index that observed the timeout
  unsigned long long epoch;
};
enum StatusCode : unsigned int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,
  kStatusBadArgument = 2,
  // A device argument check (CommDev::checks) refused a launch before any
  // memory access: `block` holds the CheckId, `rank` the offending value and
  // `epoch` the limit it broke.
  kStatusCheckFailed = 3,
};
enum CheckId : unsigned int {
  kCheckComm = 1,   // rank / world of the communicator out of range
  kCheckRoot = 2,   // root or peer index >= world
  kCheckBytes = 3,  // staged or symmetric extent beyond its buffer
  kCheckEpoch = 4,  // barrier epoch not above the one this block stored last
};

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
// Signal area at the start of every symmetric heap:
//   [0, 16K)        u64 block flags [kMaxBlocks][kMaxRanks] (collective barriers)
//   [64K, 64K+64)   u64 ready[kMaxRanks]  (fused GEMM+collective kernels: "rank r
//                   started call e", written by r into every peer)
//   [68K, 1M)       u64 tile flags [kMaxRanks][kMaxFusedTiles] (per-tile arrival)
constexpr size_t kFlagBytes = 1024 * 1024;
constexpr size_t kFusedReadyOff = 64 * 1024;
constexpr size_t kMoeDispatchDoneOff = 65 * 1024;  // u64 [kMaxRanks]: "src finished its dispatch writes"
constexpr size_t kMoeExpertDoneOff = 66 * 1024;    // u64 [kMaxRanks]: "src's expert outputs are ready"
constexpr size_t kFusedTileOff = 68 * 1024;
constexpr int kMaxFusedTiles = (int)((kFlagBytes - kFusedTileOff) / (8 * kMaxRanks));
constexpr int kThreads = 512;

struct CommDev {
  char* peer_base[kMaxRanks];
  unsigned long long* ctrl;     // local: [0] call counter, [1] finished-block count
  DeviceStatus* status;         // host-mapped status word
  unsigned long long timeout_ns;
  unsigned long long stage_off;
  unsigned long long slot_bytes;
  int rank;
  int world;
  // NVLS (NVSwitch multicast) region; null when unavailable. nvls_uc is this
  // rank's own mapping of its physical backing, nvls_mc the multicast mapping
  // through which multimem loads reduce over all ranks and multimem stores
  // reach every rank. Layout: [0, kNvlsSignalBytes) per-block signal
  // counters, then per-block staging chunks, then user allocations.
  char* nvls_uc;
  char* nvls_mc;
  unsigned long long nvls_bytes;
  unsigned int* nvls_seq;       // local per-block round counters
  // Device argument checks (NEXAR_DEVICE_CHECKS=1; compiled out with
  // -DNEXAR_NO_DEVICE_CHECKS): root / peer < world, staged and symmetric
  // extents inside their buffers, barrier epochs strictly increasing. A
  // failed check records kStatusCheckFailed and the kernel returns before
  // touching any buffer.
  int checks;
  unsigned long long heap_bytes;
};

constexpr unsigned long long kNvlsSignalBytes = 1ull << 20;
constexpr unsigned long long kNvlsChunkBytes = 512ull << 10;  // staging bytes per block per round
constexpr unsigned long long kNvlsStageBytes = (unsigned long long)kMaxBlocks * kNvlsChunkBytes;

}  // namespace nexar
