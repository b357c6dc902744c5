// C ABI of the sink-cache decode path (include/sinkcache_b200.h): argument checks, the
// split plan, workspace layout and kernel dispatch over (K type, V type, head_dim, group).
#include <atomic>
#include <climits>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include <cudaTypedefs.h>

#include "../../include/sinkcache_b200.h"
#include "sink_attend_tc.cuh"
#include "sink_kernels.cuh"
#include "sink_v2.cuh"

using namespace sinkb200;

namespace {

int elem_size(int32_t dt) {
  switch (dt) {
    case SINK_DTYPE_F32: return 4;
    case SINK_DTYPE_BF16: return 2;
    case SINK_DTYPE_F16: return 2;
    default: return 0;
  }
}

// (K storage, model dtype) pairs with kernels: fp32 or model-dtype keys, V in the model dtype.
bool supported_types(int32_t kdt, int32_t vdt) {
  if (vdt == SINK_DTYPE_BF16) return kdt == SINK_DTYPE_F32 || kdt == SINK_DTYPE_BF16;
  if (vdt == SINK_DTYPE_F16) return kdt == SINK_DTYPE_F32 || kdt == SINK_DTYPE_F16;
  if (vdt == SINK_DTYPE_F32) return kdt == SINK_DTYPE_F32;
  return false;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Plan {
  bool tc = false;       // attention on the tensor-core kernel (sink_attend_tc_kernel)
  bool cluster = false;  // stream kernel launched as one cluster of ns CTAs per pair
  int T = 0, S = 0, stage = 0, smem = 0, ctas_per_sm = 0;
  int ns = 1, rows_per_split = 0, halo_rows = 0;
  size_t off_o = 0, off_m = 0, off_l = 0, off_hk = 0, off_hv = 0, total = 256;
};

// Must agree with StreamGeom<KT, VT, D> (checked again at launch).
bool geometry(int D, int ks, int vs, Plan& pl) {
  if (D != 64 && D != 128 && D != 256) return false;
  const int lpr = D / 8, rpw = 32 / lpr;
  pl.T = 4 * kWarps * rpw;
  pl.stage = pl.T * D * (ks + vs);
  int s = kPipeBytes / pl.stage;
  pl.S = s < 2 ? 2 : (s > 4 ? 4 : s);
  pl.smem = kBarrierBytes + pl.S * pl.stage + kClusterHaloRows * D * (ks + vs);
  pl.ctas_per_sm = kSmemPerSM / (pl.smem + kSmemReservedPerCTA);
  if (pl.ctas_per_sm < 1) pl.ctas_per_sm = 1;
  return true;
}

// Attention over 16-bit K = V dtype with head_dim 128 runs on the tensor cores.
bool tc_attention(int32_t op, int32_t kdt, int32_t vdt, int D) {
  return op == SINK_OP_ATTEND && kdt == vdt && (kdt == SINK_DTYPE_BF16 || kdt == SINK_DTYPE_F16) &&
         D == kTcD;
}

void geometry_tc(Plan& pl) {
  pl.tc = true;
  pl.T = kTcRows;
  pl.S = kTcStages;
  pl.stage = kTcStageBytes;
  pl.smem = kTcSmemBytes;
  pl.ctas_per_sm = 1;
}

// Split plan: every (batch, head) pair's rows cut into `ns` items of `tps` chunks, one CTA
// each.  Regimes, from measurements over the op-bench grid on B200:
//   - a step whose pairs fit in one wave of CTAs with items of at most kMaxItemChunks
//     chunks takes exactly one wave: as many splits per pair as there are free SM slots
//     per pair (few pairs with long rows: every SM streams one long item);
//   - (stream kernel) pairs that alone fill the CTA slots, with rows that fit one item,
//     take one split each: no halo pre-pass, no combine (256 slots x 64 streams: 57.5 ->
//     43.1 us);
//   - (stream kernel) a plan of fewer than kFewWaves waves: the item size of
//     few_wave_item_chunks;
//   - otherwise items of kMinItemChunks..kMaxItemChunks chunks, aiming at kTargetWaves
//     waves, so the block scheduler evens out SMs that stream at different rates.  Items
//     shorter than 8 chunks spend too much of their time filling the pipeline (4 -> 8:
//     1,024 x 64 159.5 -> 143.8 us, 4,096 x 8 94.4 -> 87.8 us, no grid point slower).
constexpr long kMinItemChunks = 8;
constexpr long kMaxItemChunks = 32;
constexpr long kTargetWaves = 16;
// The persistent tensor-core kernel streams its items back to back, so it wants more,
// smaller items to even out the last round: about 16 per CTA.  (64 per CTA left items of
// 2 chunks at 32,768 slots x 8 streams, where each item's Q load, epilogue and partial
// cost more than the balance gained: 212 -> 184 us; no grid point slower.)
constexpr long kTcTargetItemsPerCta = 16;
constexpr long kTcMinItemChunks = 2;

// A stream-kernel plan of fewer than kFewWaves waves picks its item size by
// ceil(waves) * (chunks per item + kFillChunks): with so few waves the last one's fill
// matters, and a CTA spends about kFillChunks chunks' time filling its pipeline.  (4,096
// slots x 8 streams: 17 splits of 8 chunks, 3.7 waves, 87.8 us -> 9 splits of 15, 1.95
// waves, 79.9 us.  Over more waves the scheduler overlaps them and the model misleads.)
constexpr long kFewWaves = 4;
constexpr long kFillChunks = 3;

long few_wave_item_chunks(long pairs, long tiles, long slots, long min_chunks, long tps) {
  long best = tps, best_cost = LONG_MAX;
  for (long c = min_chunks; c <= kMaxItemChunks; ++c) {
    const long n = (tiles + c - 1) / c;
    const long waves = (pairs * n + slots - 1) / slots;
    const long cost = waves * ((tiles + n - 1) / n + kFillChunks);
    if (cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

void choose_splits(int pairs, int rows, int T, int slots, long target_waves, long min_chunks,
                   bool stream_rules, Plan& pl) {
  const long tiles = (rows + T - 1) / T;
  const long total = long(pairs) * tiles;
  long ns;
  if (long(pairs) * ((tiles + kMaxItemChunks - 1) / kMaxItemChunks) <= slots) {
    ns = slots / pairs;
  } else if (stream_rules && pairs >= slots && tiles <= kMaxItemChunks) {
    ns = 1;
  } else {
    long tps = (total + target_waves * slots - 1) / (target_waves * slots);
    tps = tps < min_chunks ? min_chunks : (tps > kMaxItemChunks ? kMaxItemChunks : tps);
    if (stream_rules && long(pairs) * ((tiles + tps - 1) / tps) < kFewWaves * slots)
      tps = few_wave_item_chunks(pairs, tiles, slots, min_chunks, tps);
    ns = (tiles + tps - 1) / tps;
  }
  if (ns > tiles) ns = tiles;
  if (ns > kMaxSplits) ns = kMaxSplits;
  if (ns < 1) ns = 1;
  const long tps = (tiles + ns - 1) / ns;  // even the items out
  pl.ns = int((tiles + tps - 1) / tps);
  pl.rows_per_split = int(tps) * T;
}

// Clustered stream-kernel launch: every split of a pair in one thread-block cluster, so the
// step is a single launch (halo rows staged in shared memory behind a cluster barrier, split
// partials merged through distributed shared memory).  Only for a step whose CTAs fit one
// wave: there it is bound by launch and memory latency, which the two extra launches of a
// split step add to; over several waves, clusters that must start together leave CTA slots
// idle (measured: 256 slots x 64 streams, 57 -> 79 us).  A one-wave plan with more than
// kClusterMax splits is cut down to kClusterMax when that adds at most kClusterExtraChunks
// chunks per split (a CTA alone on its SM takes about 2 us per chunk).  A shift of more than
// kClusterHaloRows rows keeps the halo pre-pass.
constexpr long kClusterExtraChunks = 4;

// Clusters of more than kClusterPortable CTAs only for splits of at most
// kLargeClusterChunks chunks: measured on one-wave steps with more bytes to stream, large
// clusters lose 27-31 % against the split launch (8,192 slots x 4 streams, 9 CTAs of 29
// chunks: 111.9 -> 78.5 us unclustered; 4,096 x 2, 15 of 9: 47.2 -> 34.3 us), while
// clusters of 4-5 CTAs win even with 17-26 chunk splits (2,048 x 8: 40.9 against 46.1 us).
constexpr long kClusterPortable = 8;
constexpr long kLargeClusterChunks = 4;

void choose_cluster(int pairs, int rows, int T, int slots, int drop, Plan& pl) {
  if (drop > kClusterHaloRows || pl.ns < 2) return;
  const long tiles = (rows + T - 1) / T;
  if (long(pairs) * pl.ns > slots) return;
  long ns = pl.ns, tps = pl.rows_per_split / T;
  if (ns > kClusterMax) {
    const long tps0 = tps;
    tps = (tiles + kClusterMax - 1) / kClusterMax;
    if (tps > kMaxItemChunks || tps - tps0 > kClusterExtraChunks) return;
    ns = (tiles + tps - 1) / tps;
  }
  if (ns > kClusterPortable && tps > kLargeClusterChunks) return;
  pl.ns = int(ns);
  pl.rows_per_split = int(tps) * T;
  pl.cluster = ns > 1;
}

// An in-place shift by `drop` rows copies, per split boundary, the halo rows the next split
// would overwrite first (min(drop, rows per split) rows): with splits not much longer than
// the shift, most of the window would make that round trip through the workspace (a 512-row
// shift at 4,096 slots x 8 streams took 483 us against 87 us for 16 rows).  So a shifting
// plan keeps its splits at least kHaloSplitRatio times the shift, in fewer, longer splits.
constexpr long kHaloSplitRatio = 3;

void limit_halo(int rows, int drop, Plan& pl) {
  const long want = kHaloSplitRatio * long(drop);
  if (pl.ns < 2 || pl.rows_per_split >= want) return;
  const long tiles = (rows + pl.T - 1) / pl.T;
  long tps = (want + pl.T - 1) / pl.T;
  long ns = tiles / tps;  // every split (the last one too) at least `want` rows
  if (ns < 1) ns = 1;
  tps = (tiles + ns - 1) / ns;  // even the splits out
  pl.ns = int((tiles + tps - 1) / tps);
  pl.rows_per_split = int(tps) * pl.T;
}

int32_t make_plan(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q, int32_t D,
                  int32_t kdt, int32_t vdt, int32_t rows, int32_t n_sink, int32_t window,
                  int32_t drop, int32_t num_sms, Plan& pl) {
  pl = Plan();
  if (batch < 1 || heads_kv < 1 || num_sms < 1 || num_sms > 4096) return SINK_EINVAL;
  if (long(batch) * heads_kv > (1L << 24)) return SINK_EINVAL;  // pair indices stay in int
  if (!supported_types(kdt, vdt)) return SINK_EDTYPE;
  const int ks = elem_size(kdt), vs = elem_size(vdt);
  if (!geometry(D, ks, vs, pl)) return SINK_EHEADDIM;
  if (op == SINK_OP_APPEND) return SINK_OK;
  const bool attend = op == SINK_OP_ATTEND || op == SINK_OP_FUSED_STEP;
  int G = 1;
  if (attend) {
    if (heads_q < heads_kv || heads_q % heads_kv) return SINK_EGROUP;
    G = heads_q / heads_kv;
    if (G > kMaxGroup) return SINK_EGROUP;
  }
  if (n_sink < 0 || window < 1 || drop < 0) return SINK_EINVAL;
  if (tc_attention(op, kdt, vdt, D)) geometry_tc(pl);
  int nrows;
  if (op == SINK_OP_EVICT) nrows = window;
  else if (op == SINK_OP_ATTEND || op == SINK_OP_FUSED_STEP) nrows = rows;
  else return SINK_EINVAL;
  if (nrows < 1) return SINK_EINVAL;
  const int pairs = batch * heads_kv;
  if (pl.tc)
    choose_splits(pairs, nrows, pl.T, num_sms, kTcTargetItemsPerCta, kTcMinItemChunks, false, pl);
  else {
    choose_splits(pairs, nrows, pl.T, num_sms * pl.ctas_per_sm, kTargetWaves, kMinItemChunks, true, pl);
    if (drop > 0 && (op == SINK_OP_EVICT || op == SINK_OP_FUSED_STEP)) limit_halo(nrows, drop, pl);
    choose_cluster(pairs, nrows, pl.T, num_sms * pl.ctas_per_sm, drop, pl);
  }
  // Partials and halo rows are reserved for clustered plans too: a device that cannot place
  // the cluster runs the same plan as a split launch (settle_cluster).
  size_t off = 256;  // status word
  if (attend && pl.ns > 1) {
    const size_t parts = size_t(pairs) * pl.ns * G;
    pl.off_o = off;
    off += align256(parts * D * 4);
    pl.off_m = off;
    off += align256(parts * 4);
    pl.off_l = off;
    off += align256(parts * 4);
  }
  const bool evicts = op == SINK_OP_EVICT || op == SINK_OP_FUSED_STEP;
  if (evicts && drop > 0 && pl.ns > 1) {
    pl.halo_rows = drop < pl.rows_per_split ? drop : pl.rows_per_split;
    const size_t hrows = size_t(pairs) * pl.ns * pl.halo_rows;
    pl.off_hk = off;
    off += align256(hrows * D * ks);
    pl.off_hv = off;
    off += align256(hrows * D * vs);
  }
  pl.total = off;
  return SINK_OK;
}

int device_sms(int* dev_out) {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  *dev_out = dev;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int32_t prepare_device(int dev);

int32_t check_kv(const sink_kv_buffers_t* kv) {
  if (!kv || !kv->k || !kv->v) return SINK_EINVAL;
  if (kv->batch < 1 || kv->heads_kv < 1 || kv->slots < 1) return SINK_EINVAL;
  if (!supported_types(kv->k_dtype, kv->v_dtype)) return SINK_EDTYPE;
  const int D = kv->head_dim;
  if (D != 64 && D != 128 && D != 256) return SINK_EHEADDIM;
  const int ks = elem_size(kv->k_dtype), vs = elem_size(kv->v_dtype);
  // bulk copies need 16-byte aligned row starts for every (batch, head)
  if (!aligned16(kv->k) || !aligned16(kv->v)) return SINK_ELAYOUT;
  if (((kv->k_stride_b * ks) & 15) || ((kv->k_stride_h * ks) & 15)) return SINK_ELAYOUT;
  if (((kv->v_stride_b * vs) & 15) || ((kv->v_stride_h * vs) & 15)) return SINK_ELAYOUT;
  if (kv->k_stride_b < 0 || kv->k_stride_h < 0 || kv->v_stride_b < 0 || kv->v_stride_h < 0)
    return SINK_ELAYOUT;
  return SINK_OK;
}

int32_t check_rows(const sink_rows_t* r, int32_t dtype, int32_t batch, int32_t heads, int32_t n) {
  if (!r || !r->data) return SINK_EINVAL;
  if (r->dtype != dtype) return SINK_EDTYPE;
  if (r->heads != heads || r->n != n) return SINK_EINVAL;
  (void)batch;
  return SINK_OK;
}

// Kernel launches this library has issued in the process (sink_launch_count).
std::atomic<uint64_t> g_launches{0};

cudaError_t counted(cudaError_t err) {
  if (err == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
  return err;
}

// Launch with programmatic stream serialization: the kernel may begin launching while its
// predecessor in the stream finishes (every kernel here waits on the grid dependency before
// touching memory), which hides the launch gap between the halo, stream and combine kernels.
// With cluster_x > 1 the grid is launched as clusters of cluster_x CTAs along x.
template <typename... Params, typename... Args>
int32_t launch_dependent_c(void (*kern)(Params...), dim3 grid, int threads, int smem, int cluster_x,
                           cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(cluster_x);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, args...);
  if (err != cudaSuccess) return err;
  return counted(cudaGetLastError());
}

template <typename... Params, typename... Args>
int32_t launch_dependent_n(void (*kern)(Params...), dim3 grid, int threads, int smem, cudaStream_t st,
                           Args... args) {
  return launch_dependent_c(kern, grid, threads, smem, 1, st, args...);
}

template <typename... Params, typename... Args>
int32_t launch_dependent(void (*kern)(Params...), dim3 grid, int smem, cudaStream_t st, Args... args) {
  return launch_dependent_n(kern, grid, kThreads, smem, st, args...);
}

// Warps per CTA of a clustered stream launch: 8, or 4 where the merge scratch of 8 warps
// (plus the CTA partial) does not fit the stage memory (16-bit K and V with head_dim 256).
template <typename KT, typename VT, int D, int GMAX>
constexpr int cluster_warps() {
  using Gm = StreamGeom<KT, VT, D>;
  return merge_scratch_bytes(8, GMAX, D) <= Gm::S * Gm::STAGE ? 8 : 4;
}

// Failure-detection test hook (sink_debug_fail_next_wait): armed as (chunk << 32) | polls,
// consumed by the next stream-kernel launch of the process; -1 when disarmed.
std::atomic<int64_t> g_fail_next_wait{-1};

// Cluster placement override (sink_debug_cluster_capacity): -1 asks the device; n >= 0 is
// taken as every clustered stream launch's capacity.
std::atomic<int> g_cluster_capacity_override{-1};

// How many clusters of `ns` CTAs of `kern` (threads, smem) the device holds at once, from
// cudaOccupancyMaxActiveClusters, remembered per (device, kernel, ns).  A miss while the
// stream is being captured is not queried (the launch is taken to fit, as it did eagerly).
template <typename K>
int cluster_capacity(K kern, int threads, int smem, int ns, int dev, cudaStream_t st) {
  const int forced = g_cluster_capacity_override.load(std::memory_order_relaxed);
  if (forced >= 0) return forced;
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int>, int> known;
  const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(kern), ns);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = known.find(key);
    if (it != known.end()) return it->second;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    (void)cudaGetLastError();
    return INT_MAX;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(ns));
  cfg.blockDim = dim3(unsigned(threads));
  cfg.dynamicSmemBytes = size_t(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(ns);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
    clusters = 0;
    (void)cudaGetLastError();
  }
  std::lock_guard<std::mutex> lock(mu);
  known[key] = clusters;
  return clusters;
}

// With `capacity`, nothing is launched: *capacity = how many of the plan's clusters the
// device holds at once (the plan must be clustered).
template <typename KT, typename VT, int D, int GMAX, bool ATTEND>
int32_t launch_stream(const StreamArgs& A0, const Plan& pl, int pairs, cudaStream_t st, int dev,
                      int* capacity = nullptr) {
  StreamArgs A = A0;
  using Gm = StreamGeom<KT, VT, D>;
  if (Gm::PLAN_SMEM != pl.smem || Gm::T != pl.T) return SINK_EINVAL;  // host/device geometry drift
  // clustered launches (one CTA per SM in the latency regime) run 8 warps per CTA where the
  // merge scratch of 8 warps fits the stage memory
  constexpr int NWC = cluster_warps<KT, VT, D, GMAX>();
  auto kern = pl.cluster ? sink_stream_kernel<KT, VT, D, GMAX, ATTEND, NWC> : sink_stream_kernel<KT, VT, D, GMAX, ATTEND, 4>;
  const int threads = pl.cluster ? 32 * NWC : kThreads;
  const int32_t rc = prepare_device(dev);
  if (rc) return rc;
  if (pl.cluster && (pl.ns > kClusterMax || A.cluster != 1)) return SINK_EINVAL;
  // only clustered launches stage halo rows and receive the cluster's partials in shared memory
  const int smem = pl.cluster ? Gm::SMEM : Gm::SMEM - Gm::HALO - Gm::MERGE;
  if (capacity) {
    if (!pl.cluster) return SINK_EINVAL;
    *capacity = cluster_capacity(kern, threads, smem, pl.ns, dev, st);
    return SINK_OK;
  }
  const int64_t inject = g_fail_next_wait.exchange(-1, std::memory_order_acq_rel);  // launches only
  if (inject >= 0) {
    A.skip_chunk = int(inject >> 32);
    A.wait_polls = int(inject & 0x7fffffff);
  }
  return launch_dependent_c(kern, dim3(pl.ns, pairs), threads, smem, pl.cluster ? pl.ns : 1, st, A);
}

template <bool ATTEND, typename KT, typename VT, int D>
int32_t by_group(int G, const StreamArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev, int* cap) {
  if constexpr (!ATTEND) {
    (void)G;
    return launch_stream<KT, VT, D, 1, false>(A, pl, pairs, st, dev, cap);
  } else {
    if (G <= 1) return launch_stream<KT, VT, D, 1, true>(A, pl, pairs, st, dev, cap);
    if (G <= 2) return launch_stream<KT, VT, D, 2, true>(A, pl, pairs, st, dev, cap);
    if (G <= 4) return launch_stream<KT, VT, D, 4, true>(A, pl, pairs, st, dev, cap);
    return launch_stream<KT, VT, D, 8, true>(A, pl, pairs, st, dev, cap);
  }
}

template <bool ATTEND, typename KT, typename VT>
int32_t by_dim(int D, int G, const StreamArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev, int* cap) {
  switch (D) {
    case 64: return by_group<ATTEND, KT, VT, 64>(G, A, pl, pairs, st, dev, cap);
    case 128: return by_group<ATTEND, KT, VT, 128>(G, A, pl, pairs, st, dev, cap);
    case 256: return by_group<ATTEND, KT, VT, 256>(G, A, pl, pairs, st, dev, cap);
    default: return SINK_EHEADDIM;
  }
}

template <bool ATTEND>
int32_t dispatch_stream(int kdt, int vdt, int D, int G, const StreamArgs& A, const Plan& pl,
                        int pairs, cudaStream_t st, int dev, int* cap = nullptr) {
  if (vdt == SINK_DTYPE_BF16) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, __nv_bfloat16>(D, G, A, pl, pairs, st, dev, cap);
    if (kdt == SINK_DTYPE_BF16) return by_dim<ATTEND, __nv_bfloat16, __nv_bfloat16>(D, G, A, pl, pairs, st, dev, cap);
  } else if (vdt == SINK_DTYPE_F16) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, __half>(D, G, A, pl, pairs, st, dev, cap);
    if (kdt == SINK_DTYPE_F16) return by_dim<ATTEND, __half, __half>(D, G, A, pl, pairs, st, dev, cap);
  } else if (vdt == SINK_DTYPE_F32) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, float>(D, G, A, pl, pairs, st, dev, cap);
  }
  return SINK_EDTYPE;
}

// A clustered plan runs as one wave of clusters, one per pair.  Where the device holds fewer
// of its clusters at once (cudaOccupancyMaxActiveClusters: clusters must fit a GPC, so a
// part or partition with small GPCs holds fewer than its CTA slots suggest, or none), the
// same plan runs as the split launch instead -- halo pre-pass, unclustered stream kernel,
// combine -- since clusters over several waves leave CTA slots idle.  The workspace already
// holds the split launch's partials and halo rows.
template <bool ATTEND>
int32_t settle_cluster(const sink_kv_buffers_t* kv, int G, StreamArgs& A, Plan& pl, int pairs,
                       cudaStream_t st, int dev) {
  if (!pl.cluster) return SINK_OK;
  int capacity = 0;
  const int32_t rc = dispatch_stream<ATTEND>(kv->k_dtype, kv->v_dtype, kv->head_dim, G, A, pl, pairs, st, dev,
                                             &capacity);
  if (rc) return rc;
  if (capacity < pairs) {
    pl.cluster = false;
    A.cluster = 0;
  }
  return SINK_OK;
}

template <typename VT>
int32_t launch_combine_t(int D, const StreamArgs& A, int pairs, cudaStream_t st) {
  switch (D) {
    case 64:
      return launch_dependent(sink_combine_kernel<VT, 64>, dim3(pairs, A.group * 64 / 32), 0, st, (const float*)A.o_part,
                              (const float*)A.m_part, (const float*)A.l_part, A.out, A.o_sb, A.o_sh,
                              A.heads_kv, A.group, A.ns);
    case 128:
      return launch_dependent(sink_combine_kernel<VT, 128>, dim3(pairs, A.group * 128 / 32), 0, st, (const float*)A.o_part,
                              (const float*)A.m_part, (const float*)A.l_part, A.out, A.o_sb, A.o_sh,
                              A.heads_kv, A.group, A.ns);
    case 256:
      return launch_dependent(sink_combine_kernel<VT, 256>, dim3(pairs, A.group * 256 / 32), 0, st, (const float*)A.o_part,
                              (const float*)A.m_part, (const float*)A.l_part, A.out, A.o_sb, A.o_sh,
                              A.heads_kv, A.group, A.ns);
    default: return SINK_EHEADDIM;
  }
}

int32_t launch_combine(int vdt, int D, const StreamArgs& A, int pairs, cudaStream_t st) {
  if (vdt == SINK_DTYPE_BF16) return launch_combine_t<__nv_bfloat16>(D, A, pairs, st);
  if (vdt == SINK_DTYPE_F16) return launch_combine_t<__half>(D, A, pairs, st);
  if (vdt == SINK_DTYPE_F32) return launch_combine_t<float>(D, A, pairs, st);
  return SINK_EDTYPE;
}

int32_t launch_halo(const sink_kv_buffers_t* kv, const StreamArgs& A, const Plan& pl, int pairs,
                    cudaStream_t st) {
  if (pl.ns < 2 || A.drop <= 0 || pl.cluster) return SINK_OK;
  HaloBytes H;
  const int ks = elem_size(kv->k_dtype), vs = elem_size(kv->v_dtype);
  H.k_sb = kv->k_stride_b * ks;
  H.k_sh = kv->k_stride_h * ks;
  H.v_sb = kv->v_stride_b * vs;
  H.v_sh = kv->v_stride_h * vs;
  H.krow = kv->head_dim * ks;
  H.vrow = kv->head_dim * vs;
  const long words = long(pl.ns - 1) * pl.halo_rows * ((H.krow + H.vrow) / 16);
  long cx = (words + kThreads * kHaloWordsPerThread - 1) / (kThreads * kHaloWordsPerThread);
  if (cx > 65535) cx = 65535;
  sink_halo_kernel<<<dim3(unsigned(cx), pairs), kThreads, 0, st>>>(A, H);
  return counted(cudaGetLastError());
}

void fill_common(StreamArgs& A, const sink_kv_buffers_t* kv, const Plan& pl, char* ws) {
  std::memset(&A, 0, sizeof(A));
  A.kbuf = static_cast<char*>(kv->k);
  A.vbuf = static_cast<char*>(kv->v);
  A.k_sb = kv->k_stride_b;
  A.k_sh = kv->k_stride_h;
  A.v_sb = kv->v_stride_b;
  A.v_sh = kv->v_stride_h;
  A.heads_kv = kv->heads_kv;
  A.group = 1;
  A.append_row = -1;
  A.ns = pl.ns;
  A.rows_per_split = pl.rows_per_split;
  A.halo_rows = pl.halo_rows;
  A.status = reinterpret_cast<int*>(ws);
  A.o_part = pl.off_o ? reinterpret_cast<float*>(ws + pl.off_o) : nullptr;
  A.m_part = pl.off_m ? reinterpret_cast<float*>(ws + pl.off_m) : nullptr;
  A.l_part = pl.off_l ? reinterpret_cast<float*>(ws + pl.off_l) : nullptr;
  A.halo_k = pl.off_hk ? ws + pl.off_hk : nullptr;
  A.halo_v = pl.off_hv ? ws + pl.off_hv : nullptr;
  A.cluster = pl.cluster ? 1 : 0;
  A.wait_polls = kWaitPolls;
  A.skip_chunk = -1;
}

constexpr float kLog2e = 1.4426950408889634f;

// Argument checks shared by the attention entry points, and the plan they launch with
// (everything but the workspace).
int32_t plan_attention_args(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows, void* out,
                            Plan& pl, int* dev) {
  if (!q || !q->data || !out) return SINK_EINVAL;
  if (q->dtype != kv->v_dtype) return SINK_EDTYPE;
  if (q->n != 1 || rows < 1 || rows > kv->slots) return SINK_EINVAL;
  const int sms = device_sms(dev);
  if (sms <= 0) return SINK_EDEVICE;
  return make_plan(SINK_OP_ATTEND, kv->batch, kv->heads_kv, q->heads, kv->head_dim, kv->k_dtype,
                   kv->v_dtype, rows, 0, 1, 0, sms, pl);
}

int32_t plan_attention(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows, void* out,
                       void* workspace, size_t workspace_bytes, Plan& pl, int* dev) {
  const int32_t rc = plan_attention_args(q, kv, rows, out, pl, dev);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  return SINK_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::atomic<void*> cached{nullptr};
  void* fn = cached.load(std::memory_order_acquire);
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return nullptr;
    cached.store(fn, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

// 4-D map over one cache buffer [B, Hkv, slots, 128] (innermost first), boxes of 64 columns
// x 128 rows with 128-byte swizzle; rows past `slots` read as zeros.
int32_t encode_cache_map(CUtensorMap* map, void* data, int32_t dtype, const sink_kv_buffers_t* kv,
                         int64_t stride_b, int64_t stride_h) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return SINK_EDEVICE;
  const int es = elem_size(dtype);
  const cuuint64_t dims[4] = {cuuint64_t(kv->head_dim), cuuint64_t(kv->slots), cuuint64_t(kv->heads_kv),
                              cuuint64_t(kv->batch)};
  const cuuint64_t strides[3] = {cuuint64_t(kv->head_dim) * es, cuuint64_t(stride_h) * es,
                                 cuuint64_t(stride_b) * es};
  const cuuint32_t box[4] = {64, kTcRows, 1, 1};
  const cuuint32_t unit[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, dtype == SINK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            4, data, dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SINK_OK : SINK_ELAYOUT;
}

// Persistent launch: one CTA per SM at most, each walking items (split, pair).
// 3-D map over the queries [B, Hq, 128] (the single token dimension dropped), boxes of 64
// columns x G rows (one GQA group) with 128-byte swizzle.  Fails (then the kernel loads q
// with plain loads) when q's rows are not 16-byte aligned.
int32_t encode_query_map(CUtensorMap* map, const sink_rows_t* q, int batch, int G) {
  if (!aligned16(q->data) || ((q->stride_b * 2) & 15) || ((q->stride_h * 2) & 15)) return SINK_ELAYOUT;
  if (q->stride_h < kTcD || q->stride_b < 1) return SINK_ELAYOUT;
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return SINK_EDEVICE;
  const cuuint64_t dims[3] = {cuuint64_t(kTcD), cuuint64_t(q->heads), cuuint64_t(batch)};
  const cuuint64_t strides[2] = {cuuint64_t(q->stride_h) * 2, cuuint64_t(q->stride_b) * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(G), 1};
  const cuuint32_t unit[3] = {1, 1, 1};
  const CUresult r = encode(map, q->dtype == SINK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            3, q->data, dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SINK_OK : SINK_ELAYOUT;
}

// Clusters of n tensor-core CTAs (one per SM) that fit the device at once, per device and n
// (cudaOccupancyMaxActiveClusters, queried by prepare_device outside any capture).
std::atomic<int> g_tc_clusters[64][kTcClusterMax + 1];

// A split attention whose items all run at once (one per CTA) merges its partials inside
// each pair's cluster when the device holds every such cluster together.
bool tc_cluster_merge(int dev, int ns, long items, int sms) {
  if (ns < 2 || ns > kTcClusterMax || items > sms || dev < 0 || dev >= 64) return false;
  return items / ns <= g_tc_clusters[dev][ns].load(std::memory_order_relaxed);
}

template <typename T, int GMAX>
int32_t launch_tc_g(const TcArgs& A0, const Plan& pl, int pairs, cudaStream_t st, int dev, bool* merged) {
  const bool pw = A0.place == kTcPlaceWarps;
  auto kern = pw ? sink_attend_tc_kernel<T, GMAX, true> : sink_attend_tc_kernel<T, GMAX, false>;
  const int32_t rc = prepare_device(dev);
  if (rc) return rc;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  const long items = long(pl.ns) * pairs;
  const int grid = int(items < sms ? items : sms);
  TcArgs A = A0;
  *merged = tc_cluster_merge(dev, pl.ns, items, sms);
  A.cluster = *merged ? 1 : 0;
  return launch_dependent_c(kern, dim3(grid), tc_threads(pw), kTcSmemBytes, *merged ? pl.ns : 1, st, A);
}

template <typename T>
int32_t launch_tc_t(int G, const TcArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev, bool* merged) {
  if (G <= 1) return launch_tc_g<T, 1>(A, pl, pairs, st, dev, merged);
  if (G <= 2) return launch_tc_g<T, 2>(A, pl, pairs, st, dev, merged);
  if (G <= 4) return launch_tc_g<T, 4>(A, pl, pairs, st, dev, merged);
  return launch_tc_g<T, 8>(A, pl, pairs, st, dev, merged);
}

// With `place`, the kernel runs the ring-buffer step's place work first (the v2 decode step
// in one launch).
int32_t launch_attention_tc(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows,
                            float scale, const uint8_t* mask, int64_t mask_stride_b, void* out,
                            int64_t out_stride_b, int64_t out_stride_h, void* workspace,
                            const Plan& pl, int dev, cudaStream_t st,
                            const V2PlaceArgs* place = nullptr, int place_mode = kTcPlaceNone) {
  TcArgs A;
  std::memset(&A, 0, sizeof(A));
  if (place) {
    A.place = place_mode;
    A.pa = *place;
  }
  int32_t rc = encode_cache_map(&A.kmap, kv->k, kv->k_dtype, kv, kv->k_stride_b, kv->k_stride_h);
  if (rc) return rc;
  if ((rc = encode_cache_map(&A.vmap, kv->v, kv->v_dtype, kv, kv->v_stride_b, kv->v_stride_h))) return rc;
  char* ws = static_cast<char*>(workspace);
  A.q = static_cast<const char*>(q->data);
  A.q_sb = q->stride_b;
  A.q_sh = q->stride_h;
  A.q_async = encode_query_map(&A.qmap, q, kv->batch, A.group = q->heads / kv->heads_kv) == SINK_OK;
  A.out = static_cast<char*>(out);
  A.o_sb = out_stride_b;
  A.o_sh = out_stride_h;
  A.mask = mask;
  A.mask_sb = mask_stride_b;
  A.o_part = pl.off_o ? reinterpret_cast<float*>(ws + pl.off_o) : nullptr;
  A.m_part = pl.off_m ? reinterpret_cast<float*>(ws + pl.off_m) : nullptr;
  A.l_part = pl.off_l ? reinterpret_cast<float*>(ws + pl.off_l) : nullptr;
  A.status = reinterpret_cast<int*>(ws);
  A.heads_kv = kv->heads_kv;
  A.group = q->heads / kv->heads_kv;
  A.row_end = rows;
  A.rows_per_split = pl.rows_per_split;
  A.ns = pl.ns;
  A.scale_log2 = scale * kLog2e;
  const int pairs = kv->batch * kv->heads_kv;
  A.pairs = pairs;
  bool merged = false;
  rc = kv->k_dtype == SINK_DTYPE_BF16 ? launch_tc_t<__nv_bfloat16>(A.group, A, pl, pairs, st, dev, &merged)
                                      : launch_tc_t<__half>(A.group, A, pl, pairs, st, dev, &merged);
  if (rc) return rc;
  if (pl.ns > 1 && !merged) {
    StreamArgs C;
    std::memset(&C, 0, sizeof(C));
    C.o_part = A.o_part;
    C.m_part = A.m_part;
    C.l_part = A.l_part;
    C.out = A.out;
    C.o_sb = A.o_sb;
    C.o_sh = A.o_sh;
    C.heads_kv = A.heads_kv;
    C.group = A.group;
    C.ns = A.ns;
    return launch_combine(kv->v_dtype, kv->head_dim, C, pairs, st);
  }
  return SINK_OK;
}

// Split-K decode attention over rows [0, rows): the tensor-core kernel for 16-bit K with
// head_dim 128, else the stream kernel in attend-only mode; then the split combine.
int32_t launch_attention(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows,
                         float scale, const uint8_t* mask, int64_t mask_stride_b, void* out,
                         int64_t out_stride_b, int64_t out_stride_h, void* workspace,
                         const Plan& pl, int dev, cudaStream_t st, const V2PlaceArgs* place = nullptr,
                         int place_mode = kTcPlaceNone) {
  if (pl.tc)
    return launch_attention_tc(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b,
                               out_stride_h, workspace, pl, dev, st, place, place_mode);
  if (place) return SINK_EINVAL;
  int32_t rc;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.group = q->heads / kv->heads_kv;
  A.q = static_cast<const char*>(q->data);
  A.q_sb = q->stride_b;
  A.q_sh = q->stride_h;
  A.out = static_cast<char*>(out);
  A.o_sb = out_stride_b;
  A.o_sh = out_stride_h;
  A.window = 1;
  A.row_begin = 0;
  A.row_end = rows;
  A.written_end = 0;
  A.scale_log2 = scale * kLog2e;
  A.mask = mask;
  A.mask_sb = mask_stride_b;
  const int pairs = kv->batch * kv->heads_kv;
  Plan pe = pl;
  if ((rc = settle_cluster<true>(kv, A.group, A, pe, pairs, st, dev))) return rc;
  if ((rc = dispatch_stream<true>(kv->k_dtype, kv->v_dtype, kv->head_dim, A.group, A, pe, pairs, st, dev)))
    return rc;
  if (pe.ns > 1 && !pe.cluster) return launch_combine(kv->v_dtype, kv->head_dim, A, pairs, st);
  return SINK_OK;
}

template <typename KT, typename VT>
int32_t launch_append_t(const sink_kv_buffers_t* kv, const sink_rows_t* kn, const sink_rows_t* vn,
                        int32_t row, cudaStream_t st) {
  const int64_t total = int64_t(kv->batch) * kv->heads_kv * kn->n * kv->head_dim;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  sink_append_kernel<KT, VT><<<int(blocks), threads, 0, st>>>(
      static_cast<KT*>(kv->k), static_cast<VT*>(kv->v), kv->k_stride_b, kv->k_stride_h,
      kv->v_stride_b, kv->v_stride_h, static_cast<const VT*>(kn->data),
      static_cast<const VT*>(vn->data), kn->stride_b, kn->stride_h, kn->stride_t, vn->stride_b,
      vn->stride_h, vn->stride_t, kv->heads_kv, kn->n, kv->head_dim, row, total);
  return counted(cudaGetLastError());
}


// ---------------------------------------------------------------- ring-buffer (v2) layer

bool rows_aligned16(const sink_rows_t* r, int es) {
  return aligned16(r->data) && !((r->stride_b * es) & 15) && !((r->stride_h * es) & 15);
}

// Checks of sink_v2_place / sink_v2_decode_step; fills the kernel arguments.
int32_t v2_args(const sink_kv_buffers_t* kv, const sink_rows_t* k_new, const sink_rows_t* v_new,
                const sink_rows_t* region_keys, const int64_t* region_pos, int32_t R,
                const sink_rows_t* region_out, int64_t* position, int64_t t_host, int32_t n_sink,
                int32_t window, const double* inv_freq, int32_t rot_half, V2PlaceArgs& a) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (kv->k_dtype != kv->v_dtype) return SINK_EDTYPE;
  if (n_sink < 0 || window < 1 || R < 0) return SINK_EINVAL;
  const int64_t ring = int64_t(window) + 1;
  if (ring + R > kv->slots) return SINK_EINVAL;
  if (!position && t_host < 0) return SINK_EINVAL;
  const int D = kv->head_dim, es = elem_size(kv->k_dtype);
  std::memset(&a, 0, sizeof(a));
  if ((k_new == nullptr) != (v_new == nullptr)) return SINK_EINVAL;
  if (k_new) {
    if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
    if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
    if (!rows_aligned16(k_new, es) || !rows_aligned16(v_new, es)) return SINK_ELAYOUT;
    a.knew = static_cast<const char*>(k_new->data);
    a.vnew = static_cast<const char*>(v_new->data);
    a.kn_sb = k_new->stride_b;
    a.kn_sh = k_new->stride_h;
    a.vn_sb = v_new->stride_b;
    a.vn_sh = v_new->stride_h;
  }
  a.kbuf = static_cast<char*>(kv->k);
  a.vbuf = static_cast<char*>(kv->v);
  a.k_sb = kv->k_stride_b;
  a.k_sh = kv->k_stride_h;
  a.v_sb = kv->v_stride_b;
  a.v_sh = kv->v_stride_h;
  if (R > 0) {
    if (!region_keys || !region_keys->data || !region_pos || !inv_freq) return SINK_EINVAL;
    if (region_keys->dtype != kv->k_dtype) return SINK_EDTYPE;
    if (region_keys->heads != kv->heads_kv || region_keys->n < R) return SINK_EINVAL;
    if (rot_half < 1 || 2 * rot_half > D) return SINK_EINVAL;
    a.reg_k = static_cast<const char*>(region_keys->data);
    a.rk_sb = region_keys->stride_b;
    a.rk_sh = region_keys->stride_h;
    a.rk_st = region_keys->stride_t;
    if (region_out) {
      if (!region_out->data) return SINK_EINVAL;
      if (region_out->dtype != kv->k_dtype) return SINK_EDTYPE;
      if (region_out->heads != kv->heads_kv || region_out->n < R) return SINK_EINVAL;
      a.rout = static_cast<char*>(region_out->data);
      a.ro_sb = region_out->stride_b;
      a.ro_sh = region_out->stride_h;
      a.ro_st = region_out->stride_t;
    } else {
      a.rout = static_cast<char*>(kv->k) + ring * D * es;
      a.ro_sb = kv->k_stride_b;
      a.ro_sh = kv->k_stride_h;
      a.ro_st = D;
    }
  }
  a.reg_pos = region_pos;
  a.position = position;
  a.t_host = t_host;
  a.inv_freq = inv_freq;
  a.n_sink = n_sink;
  a.window = window;
  a.ring = int(ring);
  a.R = R;
  a.rot_half = rot_half;
  a.heads_kv = kv->heads_kv;
  a.pairs = kv->batch * kv->heads_kv;
  return SINK_OK;
}

template <typename T>
int32_t launch_v2_place_t(int D, const V2PlaceArgs& a, int sms, cudaStream_t st) {
  const int grid = a.pairs < sms * 8 ? a.pairs : sms * 8;
  switch (D) {
    case 64: return launch_dependent(sink_v2_place_kernel<T, 64>, dim3(grid), 0, st, a);
    case 128: return launch_dependent(sink_v2_place_kernel<T, 128>, dim3(grid), 0, st, a);
    case 256: return launch_dependent(sink_v2_place_kernel<T, 256>, dim3(grid), 0, st, a);
    default: return SINK_EHEADDIM;
  }
}

int32_t launch_v2_place(const sink_kv_buffers_t* kv, const V2PlaceArgs& a, int sms, cudaStream_t st) {
  if (a.pairs < 1) return SINK_EINVAL;
  switch (kv->k_dtype) {
    case SINK_DTYPE_BF16: return launch_v2_place_t<__nv_bfloat16>(kv->head_dim, a, sms, st);
    case SINK_DTYPE_F16: return launch_v2_place_t<__half>(kv->head_dim, a, sms, st);
    case SINK_DTYPE_F32: return launch_v2_place_t<float>(kv->head_dim, a, sms, st);
    default: return SINK_EDTYPE;
  }
}


// ---------------------------------------------------------------- no-allocation scratch

}  // namespace

// Scratch of sink_decode_attention_noalloc.  In host code this name is only a stand-in for
// the symbol, not a device address: the host looks up each device's copy with
// cudaGetSymbolAddress and passes that pointer to the kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SINK_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch on device `dev` (the current device), looked up once
// per device: by sink_prepare_device, or by the first no-allocation call on that device.
int32_t noalloc_scratch(int dev, void** ptr) {
  static std::atomic<void*> cache[64];
  if (dev < 0 || dev >= 64) return SINK_EDEVICE;
  void* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess) return err;
    if (p == nullptr) return SINK_EDEVICE;
    cache[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  return SINK_OK;
}


// ---------------------------------------------------------------- per-device set-up

// Opt every kernel that uses more than 48 KB of dynamic shared memory into its size, and
// look up the tensor-map encoder: calls that must not happen inside a stream capture, so
// they are made once per device, by sink_prepare_device() or by the first launch.
// A kernel's dynamic shared memory, and clusters of up to 16 CTAs (above the portable 8;
// B200 schedules 16 of the stream kernel's 2-per-SM CTAs on one GPC; for the one-per-SM
// tensor-core kernel the occupancy query decides).
template <typename... Params>
cudaError_t stream_attrs(void (*kern)(Params...), int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

template <bool ATTEND, typename KT, typename VT, int D>
cudaError_t allow_smem_d() {
  const int bytes = StreamGeom<KT, VT, D>::SMEM;
  if constexpr (!ATTEND) {
    cudaError_t e = stream_attrs(sink_stream_kernel<KT, VT, D, 1, false, 4>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 1, false, cluster_warps<KT, VT, D, 1>()>, bytes);
    return e;
  } else {
    cudaError_t e = stream_attrs(sink_stream_kernel<KT, VT, D, 1, true, 4>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 2, true, 4>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 4, true, 4>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 8, true, 4>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 1, true, cluster_warps<KT, VT, D, 1>()>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 2, true, cluster_warps<KT, VT, D, 2>()>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 4, true, cluster_warps<KT, VT, D, 4>()>, bytes);
    if (e == cudaSuccess) e = stream_attrs(sink_stream_kernel<KT, VT, D, 8, true, cluster_warps<KT, VT, D, 8>()>, bytes);
    return e;
  }
}

template <bool ATTEND, typename KT, typename VT>
cudaError_t allow_smem_t() {
  cudaError_t e = allow_smem_d<ATTEND, KT, VT, 64>();
  if (e == cudaSuccess) e = allow_smem_d<ATTEND, KT, VT, 128>();
  if (e == cudaSuccess) e = allow_smem_d<ATTEND, KT, VT, 256>();
  return e;
}

template <bool ATTEND>
cudaError_t allow_smem_stream() {
  cudaError_t e = allow_smem_t<ATTEND, float, __nv_bfloat16>();
  if (e == cudaSuccess) e = allow_smem_t<ATTEND, __nv_bfloat16, __nv_bfloat16>();
  if (e == cudaSuccess) e = allow_smem_t<ATTEND, float, __half>();
  if (e == cudaSuccess) e = allow_smem_t<ATTEND, __half, __half>();
  if (e == cudaSuccess) e = allow_smem_t<ATTEND, float, float>();
  return e;
}

template <typename T>
cudaError_t allow_smem_tc() {
  const int b = kTcSmemBytes;
  cudaError_t e = stream_attrs(sink_attend_tc_kernel<T, 1, false>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 2, false>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 4, false>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 8, false>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 1, true>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 2, true>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 4, true>, b);
  if (e == cudaSuccess) e = stream_attrs(sink_attend_tc_kernel<T, 8, true>, b);
  return e;
}

std::atomic<uint64_t> g_prepared{0};  // one bit per device

// How many clusters of n tensor-core CTAs the device holds at once (0 when the query fails:
// that size is then never clustered).
void tc_cluster_capacity(int dev) {
  if (dev < 0 || dev >= 64) return;
  for (int n = 2; n <= kTcClusterMax; ++n) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(n));
    cfg.blockDim = dim3(tc_threads(false));
    cfg.dynamicSmemBytes = kTcSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(n);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, sink_attend_tc_kernel<__nv_bfloat16, 2, false>, &cfg) != cudaSuccess) {
      clusters = 0;
      (void)cudaGetLastError();
    }
    g_tc_clusters[dev][n].store(clusters, std::memory_order_relaxed);
  }
}

int32_t prepare_device(int dev) {
  const uint64_t bit = uint64_t(1) << dev;
  if (g_prepared.load(std::memory_order_acquire) & bit) return SINK_OK;
  cudaError_t e = allow_smem_stream<false>();
  if (e == cudaSuccess) e = allow_smem_stream<true>();
  if (e == cudaSuccess) e = allow_smem_tc<__nv_bfloat16>();
  if (e == cudaSuccess) e = allow_smem_tc<__half>();
  if (e != cudaSuccess) return e;
  tc_cluster_capacity(dev);
  if (tensor_map_encoder() == nullptr) return SINK_EDEVICE;
  void* scratch = nullptr;  // the no-allocation entry point's static array, on this device
  const int32_t rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  g_prepared.fetch_or(bit, std::memory_order_acq_rel);
  return SINK_OK;
}

}  // namespace

extern "C" {

int32_t sink_abi_version(void) { return SINK_ABI_VERSION; }

uint64_t sink_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* sink_strerror(int32_t code) {
  switch (code) {
    case SINK_OK: return "ok";
    case SINK_EINVAL: return "sinkcache_b200: size or index out of range";
    case SINK_EDTYPE: return "sinkcache_b200: unsupported dtype combination (K fp32 or model dtype; V, q, new rows in the model dtype bf16/fp16/fp32)";
    case SINK_EHEADDIM: return "sinkcache_b200: head_dim must be 64, 128 or 256";
    case SINK_EGROUP: return "sinkcache_b200: heads_q / heads_kv must be an integer between 1 and 8";
    case SINK_ELAYOUT: return "sinkcache_b200: cache rows must be contiguous and 16-byte aligned";
    case SINK_EWORKSPACE: return "sinkcache_b200: workspace missing or smaller than sink_workspace_bytes()";
    case SINK_EDEVICE: return "sinkcache_b200: no usable CUDA device";
    case SINK_ESCRATCH: return "sinkcache_b200: request needs more than the 16 MiB static scratch of sink_decode_attention_noalloc; use sink_decode_attention with a workspace";
    default:
      if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
      return "sinkcache_b200: unknown error";
  }
}

size_t sink_workspace_bytes(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q,
                            int32_t head_dim, int32_t k_dtype, int32_t v_dtype, int32_t rows,
                            int32_t n_sink, int32_t window, int32_t drop, int32_t num_sms) {
  Plan pl;
  if (make_plan(op, batch, heads_kv, heads_q, head_dim, k_dtype, v_dtype, rows, n_sink, window,
                drop, num_sms, pl) != SINK_OK)
    return 0;
  return pl.total;
}

int32_t sink_plan(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q, int32_t head_dim,
                  int32_t k_dtype, int32_t v_dtype, int32_t rows, int32_t n_sink, int32_t window,
                  int32_t drop, int32_t num_sms, int32_t* splits, int32_t* rows_per_split,
                  int32_t* chunk_rows, int32_t* stages, int32_t* smem_bytes,
                  int32_t* cluster_ctas) {
  Plan pl;
  const int32_t rc = make_plan(op, batch, heads_kv, heads_q, head_dim, k_dtype, v_dtype, rows,
                               n_sink, window, drop, num_sms, pl);
  if (rc != SINK_OK) return rc;
  if (splits) *splits = pl.ns;
  if (rows_per_split) *rows_per_split = pl.rows_per_split;
  if (chunk_rows) *chunk_rows = pl.T;
  if (stages) *stages = pl.S;
  if (smem_bytes) *smem_bytes = pl.smem;
  if (cluster_ctas) *cluster_ctas = pl.cluster ? pl.ns : 1;
  return SINK_OK;
}

int32_t sink_plan_launch(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q,
                         int32_t head_dim, int32_t k_dtype, int32_t v_dtype, int32_t rows,
                         int32_t n_sink, int32_t window, int32_t drop, int32_t num_sms,
                         int32_t* mode, int32_t* ctas) {
  Plan pl;
  const int32_t rc = make_plan(op, batch, heads_kv, heads_q, head_dim, k_dtype, v_dtype, rows,
                               n_sink, window, drop, num_sms, pl);
  if (rc != SINK_OK) return rc;
  const long items = long(batch) * heads_kv * pl.ns;
  int m = SINK_LAUNCH_SPLIT;
  long n = items;
  if (pl.tc) {
    m = SINK_LAUNCH_TENSOR;
    n = items < num_sms ? items : num_sms;
  } else if (pl.cluster) {
    m = SINK_LAUNCH_CLUSTER;
  }
  if (op == SINK_OP_APPEND) n = 0;
  if (mode) *mode = m;
  if (ctas) *ctas = int32_t(n);
  return SINK_OK;
}

int32_t sink_append(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                    const sink_rows_t* v_new, int32_t row, void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, k_new ? k_new->n : 0))) return rc;
  if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, k_new->n))) return rc;
  if (k_new->n < 1 || row < 0 || row + k_new->n > kv->slots) return SINK_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kdt = kv->k_dtype, vdt = kv->v_dtype;
  if (vdt == SINK_DTYPE_BF16) {
    if (kdt == SINK_DTYPE_F32) return launch_append_t<float, __nv_bfloat16>(kv, k_new, v_new, row, st);
    return launch_append_t<__nv_bfloat16, __nv_bfloat16>(kv, k_new, v_new, row, st);
  }
  if (vdt == SINK_DTYPE_F16) {
    if (kdt == SINK_DTYPE_F32) return launch_append_t<float, __half>(kv, k_new, v_new, row, st);
    return launch_append_t<__half, __half>(kv, k_new, v_new, row, st);
  }
  return launch_append_t<float, float>(kv, k_new, v_new, row, st);
}

}  // extern "C"

namespace {

// sink_evict_rerotate, and with `kc` the variant that also writes every window row's final
// key, in the value type, into kc (then drop == 0 launches too: a pure conversion).
int32_t evict_launch(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window, int32_t drop,
                     const float* cos_tab, const float* sin_tab, int32_t rotate,
                     const sink_rows_t* kc, void* workspace, size_t workspace_bytes,
                     void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (n_sink < 0 || window < 1 || drop < 0) return SINK_EINVAL;
  if (int64_t(n_sink) + window + drop > kv->slots) return SINK_EINVAL;
  if (kc) {
    if ((rc = check_rows(kc, kv->v_dtype, kv->batch, kv->heads_kv, kc->n))) return rc;
    if (kc->n < n_sink + window || kc->stride_t != kv->head_dim) return SINK_ELAYOUT;
    if (!rows_aligned16(kc, elem_size(kv->v_dtype))) return SINK_ELAYOUT;
  }
  if (drop == 0 && !kc) return SINK_OK;
  if (drop > 0 && rotate && (!cos_tab || !sin_tab)) return SINK_EINVAL;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_EVICT, kv->batch, kv->heads_kv, kv->heads_kv, kv->head_dim, kv->k_dtype,
                 kv->v_dtype, 0, n_sink, window, drop, sms, pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.n_sink = n_sink;
  A.window = window;
  A.drop = drop;
  A.rotate = rotate ? 1 : 0;
  A.cos_tab = cos_tab;
  A.sin_tab = sin_tab;
  A.row_begin = n_sink;
  A.row_end = n_sink + window;
  A.written_end = n_sink + window;
  if (kc) {
    A.kmirror = static_cast<char*>(kc->data);
    A.km_sb = kc->stride_b;
    A.km_sh = kc->stride_h;
  }
  const int pairs = kv->batch * kv->heads_kv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = settle_cluster<false>(kv, 1, A, pl, pairs, st, dev))) return rc;
  if ((rc = launch_halo(kv, A, pl, pairs, st))) return rc;
  return dispatch_stream<false>(kv->k_dtype, kv->v_dtype, kv->head_dim, 1, A, pl, pairs, st, dev);
}

}  // namespace

extern "C" {

int32_t sink_evict_rerotate(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                            int32_t drop, const float* cos_tab, const float* sin_tab,
                            int32_t rotate, void* workspace, size_t workspace_bytes,
                            void* stream) {
  return evict_launch(kv, n_sink, window, drop, cos_tab, sin_tab, rotate, nullptr, workspace,
                      workspace_bytes, stream);
}

int32_t sink_evict_rerotate_keycopy(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                                    int32_t drop, const float* cos_tab, const float* sin_tab,
                                    int32_t rotate, const sink_rows_t* k_copy, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!k_copy) return SINK_EINVAL;
  return evict_launch(kv, n_sink, window, drop, cos_tab, sin_tab, rotate, k_copy, workspace,
                      workspace_bytes, stream);
}

int32_t sink_decode_attention(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows,
                              float scale, const uint8_t* mask, int64_t mask_stride_b,
                              void* out, int64_t out_stride_b, int64_t out_stride_h,
                              void* workspace, size_t workspace_bytes, void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  Plan pl;
  int dev = 0;
  if ((rc = plan_attention(q, kv, rows, out, workspace, workspace_bytes, pl, &dev))) return rc;
  return launch_attention(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b,
                          out_stride_h, workspace, pl, dev, static_cast<cudaStream_t>(stream));
}

int32_t sink_fused_decode_step(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                               const sink_rows_t* v_new, const sink_rows_t* q,
                               int32_t n_sink, int32_t window, int32_t drop,
                               int32_t append_row, const float* cos_tab, const float* sin_tab,
                               int32_t rotate, float scale, const uint8_t* mask,
                               int64_t mask_stride_b, void* out, int64_t out_stride_b,
                               int64_t out_stride_h, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
  if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
  if (!q || !q->data || !out) return SINK_EINVAL;
  if (q->dtype != kv->v_dtype) return SINK_EDTYPE;
  if (q->n != 1) return SINK_EINVAL;
  if (n_sink < 0 || window < 1 || drop < 0 || append_row < 0 || append_row >= kv->slots)
    return SINK_EINVAL;
  if (drop > 0) {
    if (append_row != n_sink + window) return SINK_EINVAL;
    if (int64_t(n_sink) + window + drop > kv->slots) return SINK_EINVAL;
    if (rotate && (!cos_tab || !sin_tab)) return SINK_EINVAL;
  }
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_FUSED_STEP, kv->batch, kv->heads_kv, q->heads, kv->head_dim,
                 kv->k_dtype, kv->v_dtype, append_row + 1, n_sink, window, drop, sms, pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.group = q->heads / kv->heads_kv;
  A.knew = static_cast<const char*>(k_new->data);
  A.vnew = static_cast<const char*>(v_new->data);
  A.kn_sb = k_new->stride_b;
  A.kn_sh = k_new->stride_h;
  A.vn_sb = v_new->stride_b;
  A.vn_sh = v_new->stride_h;
  A.q = static_cast<const char*>(q->data);
  A.q_sb = q->stride_b;
  A.q_sh = q->stride_h;
  A.out = static_cast<char*>(out);
  A.o_sb = out_stride_b;
  A.o_sh = out_stride_h;
  A.cos_tab = cos_tab;
  A.sin_tab = sin_tab;
  A.n_sink = n_sink;
  A.window = window;
  A.drop = drop;
  A.rotate = rotate ? 1 : 0;
  A.row_begin = 0;
  A.row_end = append_row + 1;
  A.append_row = append_row;
  A.written_end = drop > 0 ? n_sink + window + 1 : append_row + 1;
  A.scale_log2 = scale * kLog2e;
  A.mask = mask;
  A.mask_sb = mask_stride_b;
  const int pairs = kv->batch * kv->heads_kv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = settle_cluster<true>(kv, A.group, A, pl, pairs, st, dev))) return rc;
  if ((rc = launch_halo(kv, A, pl, pairs, st))) return rc;
  if ((rc = dispatch_stream<true>(kv->k_dtype, kv->v_dtype, kv->head_dim, A.group, A, pl, pairs, st, dev)))
    return rc;
  if (pl.ns > 1 && !pl.cluster) return launch_combine(kv->v_dtype, kv->head_dim, A, pairs, st);
  return SINK_OK;
}

int32_t sink_v2_place(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                      const sink_rows_t* v_new, const sink_rows_t* region_keys,
                      const int64_t* region_pos, int32_t region_len,
                      const sink_rows_t* region_out, int64_t* position, int64_t t_host,
                      int32_t n_sink, int32_t window, const double* inv_freq,
                      int32_t rot_half, void* stream) {
  V2PlaceArgs a;
  const int32_t rc = v2_args(kv, k_new, v_new, region_keys, region_pos, region_len, region_out,
                             position, t_host, n_sink, window, inv_freq, rot_half, a);
  if (rc) return rc;
  if (!k_new && region_len == 0 && !position) return SINK_OK;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  return launch_v2_place(kv, a, sms, static_cast<cudaStream_t>(stream));
}

constexpr long kPlaceWarpsChunksPerCta = 16;

int32_t sink_v2_decode_step(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                            const sink_rows_t* v_new, const sink_rows_t* region_keys,
                            const int64_t* region_pos, int32_t region_len, int64_t* position,
                            int32_t n_sink, int32_t window, const double* inv_freq,
                            int32_t rot_half, const sink_rows_t* q, float scale,
                            const uint8_t* mask, int64_t mask_stride_b, void* out,
                            int64_t out_stride_b, int64_t out_stride_h, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!k_new || !position) return SINK_EINVAL;
  V2PlaceArgs a;
  int32_t rc = v2_args(kv, k_new, v_new, region_keys, region_pos, region_len, nullptr, position,
                       0, n_sink, window, inv_freq, rot_half, a);
  if (rc) return rc;
  const int32_t rows = window + 1 + region_len;
  Plan pl;
  int dev = 0;
  if ((rc = plan_attention(q, kv, rows, out, workspace, workspace_bytes, pl, &dev))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  // One launch on the tensor-core path, each CTA placing the rows of its own items.  Long
  // steps whose CTAs walk several items (at least kPlaceWarpsChunksPerCta chunks per CTA):
  // two warps place item by item beside the pipeline, which waits only for the chunks
  // holding placed rows.  Other steps with no more pairs than SMs: every thread places
  // before the pipeline starts; split-major items put each pair's region and new-token items
  // on different CTAs.  Short steps over more pairs keep the place kernel (one CTA per pair)
  // before the attention: there a CTA would place several pairs' region rows on the step's
  // critical path.
  if (pl.tc) {
    const long items = long(a.pairs) * pl.ns;
    const long ctas = items < sms ? items : sms;
    const long chunks = long(a.pairs) * ((rows + kTcRows - 1) / kTcRows);
    int mode = kTcPlaceNone;
    if (items > ctas && chunks >= kPlaceWarpsChunksPerCta * ctas) mode = kTcPlaceWarps;
    else if (a.pairs <= sms) mode = kTcPlaceFirst;
    if (mode != kTcPlaceNone)
      return launch_attention(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b,
                              out_stride_h, workspace, pl, dev, st, &a, mode);
  }
  if ((rc = launch_v2_place(kv, a, sms, st))) return rc;
  return launch_attention(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b,
                          out_stride_h, workspace, pl, dev, st);
}

int32_t sink_debug_cluster_capacity(int32_t clusters) {
  if (clusters < -1) return SINK_EINVAL;
  g_cluster_capacity_override.store(clusters, std::memory_order_relaxed);
  return SINK_OK;
}

int32_t sink_debug_fail_next_wait(int32_t chunk, int32_t polls) {
  if (chunk < 0 || polls < 1) return SINK_EINVAL;
  g_fail_next_wait.store((int64_t(chunk) << 32) | int64_t(polls), std::memory_order_release);
  return SINK_OK;
}

int32_t sink_v2_gather(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                       int32_t region_len, int64_t lo, int64_t hi, const sink_rows_t* k_new,
                       const sink_rows_t* v_new, const sink_rows_t* out_k, const sink_rows_t* out_v,
                       void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (kv->k_dtype != kv->v_dtype) return SINK_EDTYPE;
  const int es = elem_size(kv->k_dtype);
  if (n_sink < 0 || window < 1 || region_len < 0) return SINK_EINVAL;
  const int64_t ring = int64_t(window) + 1;
  if (ring + region_len > kv->slots) return SINK_EINVAL;
  const int64_t nwin = hi > lo ? hi - lo : 0;
  if (nwin > 0 && (lo < n_sink || nwin > ring)) return SINK_EINVAL;
  if ((k_new == nullptr) != (v_new == nullptr)) return SINK_EINVAL;
  const int n = k_new ? k_new->n : 0;
  if (k_new) {
    if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, n))) return rc;
    if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, n))) return rc;
    if (!rows_aligned16(k_new, es) || !rows_aligned16(v_new, es) || ((k_new->stride_t * es) & 15) ||
        ((v_new->stride_t * es) & 15))
      return SINK_ELAYOUT;
  }
  const int64_t rows = region_len + nwin + n;
  if (rows > INT_MAX) return SINK_EINVAL;
  if (!out_k || !out_v) return SINK_EINVAL;
  if ((rc = check_rows(out_k, kv->k_dtype, kv->batch, kv->heads_kv, out_k->n))) return rc;
  if ((rc = check_rows(out_v, kv->v_dtype, kv->batch, kv->heads_kv, out_v->n))) return rc;
  if (out_k->n < rows || out_v->n < rows) return SINK_EINVAL;
  if (!rows_aligned16(out_k, es) || !rows_aligned16(out_v, es) || ((out_k->stride_t * es) & 15) ||
      ((out_v->stride_t * es) & 15))
    return SINK_ELAYOUT;
  if (rows == 0) return SINK_OK;
  V2GatherArgs g;
  std::memset(&g, 0, sizeof(g));
  g.kbuf = static_cast<const char*>(kv->k);
  g.vbuf = static_cast<const char*>(kv->v);
  g.k_sb = kv->k_stride_b;
  g.k_sh = kv->k_stride_h;
  g.v_sb = kv->v_stride_b;
  g.v_sh = kv->v_stride_h;
  if (k_new) {
    g.knew = static_cast<const char*>(k_new->data);
    g.vnew = static_cast<const char*>(v_new->data);
    g.kn_sb = k_new->stride_b;
    g.kn_sh = k_new->stride_h;
    g.kn_st = k_new->stride_t;
    g.vn_sb = v_new->stride_b;
    g.vn_sh = v_new->stride_h;
    g.vn_st = v_new->stride_t;
  }
  g.ok = static_cast<char*>(out_k->data);
  g.ov = static_cast<char*>(out_v->data);
  g.ok_sb = out_k->stride_b;
  g.ok_sh = out_k->stride_h;
  g.ok_st = out_k->stride_t;
  g.ov_sb = out_v->stride_b;
  g.ov_sh = out_v->stride_h;
  g.ov_st = out_v->stride_t;
  g.lo = lo;
  g.n_sink = n_sink;
  g.ring = int(ring);
  g.R = region_len;
  g.nwin = int(nwin);
  g.n = n;
  g.rows = int(rows);
  g.heads_kv = kv->heads_kv;
  g.pairs = kv->batch * kv->heads_kv;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  const long long words = 2LL * g.pairs * rows * (kv->head_dim * es / 16);
  long long grid = (words + kThreads * kGatherWordsPerThread - 1) / (kThreads * kGatherWordsPerThread);
  if (grid > 8LL * sms) grid = 8LL * sms;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kern) { return launch_dependent(kern, dim3(unsigned(grid)), 0, st, g); };
  switch (kv->k_dtype) {
    case SINK_DTYPE_BF16:
      if (kv->head_dim == 64) return go(sink_v2_gather_kernel<__nv_bfloat16, 64>);
      if (kv->head_dim == 128) return go(sink_v2_gather_kernel<__nv_bfloat16, 128>);
      return go(sink_v2_gather_kernel<__nv_bfloat16, 256>);
    case SINK_DTYPE_F16:
      if (kv->head_dim == 64) return go(sink_v2_gather_kernel<__half, 64>);
      if (kv->head_dim == 128) return go(sink_v2_gather_kernel<__half, 128>);
      return go(sink_v2_gather_kernel<__half, 256>);
    case SINK_DTYPE_F32:
      if (kv->head_dim == 64) return go(sink_v2_gather_kernel<float, 64>);
      if (kv->head_dim == 128) return go(sink_v2_gather_kernel<float, 128>);
      return go(sink_v2_gather_kernel<float, 256>);
    default: return SINK_EDTYPE;
  }
}

int32_t sink_prepare_device(void) {
  int dev = 0;
  if (device_sms(&dev) <= 0) return SINK_EDEVICE;
  return prepare_device(dev);
}

int32_t sink_read_status(void* workspace, void* stream, int32_t* status) {
  if (!workspace || !status) return SINK_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  cudaError_t err = cudaMemcpyAsync(&host, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err == cudaSuccess) err = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  *status = host;
  return err;
}

}  // extern "C"

extern "C" int32_t sink_decode_attention_noalloc(const sink_rows_t* q, const sink_kv_buffers_t* kv,
                                                 int32_t rows, float scale, const uint8_t* mask,
                                                 int64_t mask_stride_b, void* out,
                                                 int64_t out_stride_b, int64_t out_stride_h,
                                                 void* stream) {
  // Every argument check of sink_decode_attention runs first, so a bad request returns the
  // same code as there and launches nothing; only then the scratch size.
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  Plan pl;
  int dev = 0;
  if ((rc = plan_attention_args(q, kv, rows, out, pl, &dev))) return rc;
  if (pl.total > SINK_NOALLOC_SCRATCH_BYTES) return SINK_ESCRATCH;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(dev, &scratch))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t err = cudaMemsetAsync(scratch, 0, sizeof(int32_t), st);  // status word
  if (err != cudaSuccess) return err;
  return launch_attention(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b, out_stride_h,
                          scratch, pl, dev, st);
}
