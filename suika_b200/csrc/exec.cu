// Device executor of the B200 live-reshard path (sm_100a), C ABI in include/suika_reshard.h.
//
// One launch runs a whole copy table for one target rank. Each entry is a strided copy
// (rows x row_bytes, independent source and target pitches) whose source is either this GPU's
// HBM or a peer GPU's HBM mapped through CUDA IPC, so a single kernel does what the reference
// spreads over per-tensor NCCL isend/irecv, chunk().contiguous() and torch.cat/clone
// (Suika/migration.py:310,466,489,501,536-538; Suika/utils.py:212-236).
//
// Work decomposition: every entry is cut into tiles of about kTileBytes (whole rows when rows
// are short, column chunks of one row when rows are long); the tile list is implicit (a prefix
// of tile counts per entry, binary-searched by each CTA). CTAs stride over tiles; a CTA moves a
// tile with 16-byte vector loads/stores (narrower only when an address or pitch is not 16-byte
// aligned), several loads in flight per thread before their stores, which keeps enough bytes
// outstanding to cover NVLink read latency as well as HBM latency.
//
// Two TMA kernels run the same tables: a bulk copy (cp.async.bulk, one request per row) and a
// tensor-map copy (cp.async.bulk.tensor.3d boxes of whole rows) that takes the wide local rows of
// a one-GPU relayout. The copy is pure data movement: no tensor cores, and no TMA multicast (this
// code runs on several GPUs). The vector kernel has no waits; the TMA kernels' mbarrier waits are
// bounded by %globaltimer and report a timeout in the table's status word.
#include "../../include/suika_reshard.h"
#include "internal.h"

#include <cuda_runtime.h>
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unistd.h>
#include <vector>

namespace {

int efail(int code, const std::string& msg) { return suika_rs::fail(code, msg); }

int cuda_fail(cudaError_t e, const char* what) {
  return efail(RS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

// One table entry as the kernel reads it (72 bytes).
struct DevSeg {
  uint64_t src;
  uint64_t dst;
  uint64_t src_pitch;
  uint64_t dst_pitch;
  uint64_t tile_begin;   // global index of this entry's first tile
  uint64_t row_bytes;
  uint64_t col_bytes;    // bytes of one column chunk when rows are split, else row_bytes
  uint32_t rows;
  uint32_t rows_per_tile;
  uint32_t col_tiles;    // column chunks per row (1 when whole rows fit in a tile)
  uint32_t vshift;       // log2 of the vector width (0..4)
};
static_assert(sizeof(DevSeg) == 72, "DevSeg layout");

constexpr uint64_t kDefaultTileBytes = 128 * 1024;

template <int VB> struct Vec;
template <> struct Vec<16> { using T = uint4; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<2> { using T = uint16_t; };
template <> struct Vec<1> { using T = uint8_t; };

// Source reads bypass L1 allocation (each byte is read once); the source is not written while
// the kernel runs.
__device__ __forceinline__ uint4 load_vec(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 load_vec(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t load_vec(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t load_vec(const uint16_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ uint8_t load_vec(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned char*>(p)); }

// Streaming variant: the target is written once (.cs: evict-first store), for copies far larger
// than L2. (An L2 eviction hint on 16-byte loads does not assemble for sm_100a.)
__device__ __forceinline__ uint4 load_vec_stream(const uint4* p) { return load_vec(p); }
__device__ __forceinline__ void store_vec_stream(uint4* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void store_vec(uint4* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void store_vec(uint2* p, const uint2& v) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void store_vec(uint32_t* p, const uint32_t& v) { *p = v; }
__device__ __forceinline__ void store_vec(uint16_t* p, const uint16_t& v) { *p = v; }
__device__ __forceinline__ void store_vec(uint8_t* p, const uint8_t& v) { *p = v; }

template <bool STREAM> __device__ __forceinline__ uint4 load16(const uint4* p) { return STREAM ? load_vec_stream(p) : load_vec(p); }
template <bool STREAM> __device__ __forceinline__ void store16(uint4* p, const uint4& v) {
  if (STREAM) store_vec_stream(p, v); else store_vec(p, v);
}

// 16-byte rectangle copy with optional streaming hints (same structure as copy_rect below).
template <int U, bool STREAM>
__device__ __forceinline__ void copy_rect16(const char* __restrict__ src, char* __restrict__ dst, uint32_t nr, uint32_t vpr,
                                            uint64_t sp, uint64_t dp) {
  const uint32_t total = nr * vpr;
  const uint32_t stride = blockDim.x;
  if (nr == 1) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (uint32_t base = threadIdx.x; base < total; base += stride * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = base + u * stride;
        if (i < total) v[u] = load16<STREAM>(s + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = base + u * stride;
        if (i < total) store16<STREAM>(d + i, v[u]);
      }
    }
    return;
  }
  const uint32_t sp32 = (uint32_t)sp, dp32 = (uint32_t)dp;
  for (uint32_t base = threadIdx.x; base < total; base += stride * U) {
    uint4 v[U];
    uint32_t doff[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) {
        const uint32_t r = i / vpr;
        const uint32_t cb = (i - r * vpr) * 16;
        v[u] = load16<STREAM>(reinterpret_cast<const uint4*>(src + (r * sp32 + cb)));
        doff[u] = r * dp32 + cb;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) store16<STREAM>(reinterpret_cast<uint4*>(dst + doff[u]), v[u]);
    }
  }
}

// Copy an nr x (vpr * VB bytes) rectangle. U loads are issued before their stores. In a
// multi-row rectangle every in-tile offset fits 32 bits (the host caps rows per tile so that
// (nr - 1) * max(sp, dp) + row bytes < 2^32), which keeps the per-load state small.
template <int VB, int U>
__device__ __forceinline__ void copy_rect(const char* __restrict__ src, char* __restrict__ dst, uint32_t nr,
                                          uint32_t vpr, uint64_t sp, uint64_t dp) {
  using V = typename Vec<VB>::T;
  const uint32_t total = nr * vpr;
  const uint32_t stride = blockDim.x;
  if (nr == 1) {
    const V* s = reinterpret_cast<const V*>(src);
    V* d = reinterpret_cast<V*>(dst);
    for (uint32_t base = threadIdx.x; base < total; base += stride * U) {
      V v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = base + u * stride;
        if (i < total) v[u] = load_vec(s + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = base + u * stride;
        if (i < total) store_vec(d + i, v[u]);
      }
    }
    return;
  }
  const uint32_t sp32 = (uint32_t)sp, dp32 = (uint32_t)dp;
  for (uint32_t base = threadIdx.x; base < total; base += stride * U) {
    V v[U];
    uint32_t doff[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) {
        const uint32_t r = i / vpr;
        const uint32_t cb = (i - r * vpr) * VB;
        v[u] = load_vec(reinterpret_cast<const V*>(src + (r * sp32 + cb)));
        doff[u] = r * dp32 + cb;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) store_vec(reinterpret_cast<V*>(dst + doff[u]), v[u]);
    }
  }
}

// Tile scheduling shared by the kernels. The table holds the remote entries first (tiles
// [0, n_remote)) and the local ones after them (tiles [n_remote, n_tiles)). CTA b visits tiles
// b, b + grid, b + 2 grid, ... of each range and interleaves the two in proportion to their
// counts, so NVLink and HBM copies overlap inside every CTA instead of running one after the
// other. Tile indices only grow within a range, so each cursor finds its entry with one binary
// search and a forward walk.
struct TileCursor {
  uint64_t t, end, next_begin;
  int32_t si;
  __device__ void init(const DevSeg* __restrict__ segs, int32_t nseg, uint64_t first, uint64_t end_) {
    t = first;
    end = end_;
    si = 0;
    next_begin = ~0ull;
    if (t >= end) return;
    int32_t lo = 0, hi = nseg - 1;
    while (lo < hi) {
      const int32_t mid = (lo + hi + 1) >> 1;
      if (segs[mid].tile_begin <= t) lo = mid; else hi = mid - 1;
    }
    si = lo;
    next_begin = (si + 1 < nseg) ? segs[si + 1].tile_begin : ~0ull;
  }
  __device__ const DevSeg& locate(const DevSeg* __restrict__ segs, int32_t nseg) {
    while (t >= next_begin) {
      ++si;
      next_begin = (si + 1 < nseg) ? segs[si + 1].tile_begin : ~0ull;
    }
    return segs[si];
  }
};

struct Tile {
  const char* src;
  char* dst;
  uint64_t sp, dp, nb;
  uint32_t nr, vshift;
};

__device__ __forceinline__ Tile tile_of(const DevSeg& s, uint64_t t) {
  Tile x;
  const uint64_t lt = t - s.tile_begin;
  const uint64_t rg = lt / s.col_tiles;
  const uint64_t col = lt - rg * s.col_tiles;
  const uint64_t r0 = rg * s.rows_per_tile;
  x.nr = (uint32_t)min((uint64_t)s.rows_per_tile, (uint64_t)s.rows - r0);
  const uint64_t c0 = col * s.col_bytes;
  x.nb = min(s.col_bytes, s.row_bytes - c0);
  x.sp = s.src_pitch;
  x.dp = s.dst_pitch;
  x.src = reinterpret_cast<const char*>(s.src) + r0 * x.sp + c0;
  x.dst = reinterpret_cast<char*>(s.dst) + r0 * x.dp + c0;
  x.vshift = s.vshift;
  return x;
}

struct Schedule {
  TileCursor rc, lc;
  uint64_t n_r, n_l, d_r, d_l;
  __device__ void init(const DevSeg* __restrict__ segs, int32_t nseg, uint64_t ntiles, uint64_t nremote) {
    const uint64_t b = blockIdx.x, g = gridDim.x;
    rc.init(segs, nseg, b, nremote);
    lc.init(segs, nseg, nremote + b, ntiles);
    n_r = nremote > b ? (nremote - b + g - 1) / g : 0;
    n_l = ntiles - nremote > b ? (ntiles - nremote - b + g - 1) / g : 0;
    d_r = d_l = 0;
  }
  __device__ bool next(const DevSeg* __restrict__ segs, int32_t nseg, Tile& out) {
    const bool hr = d_r < n_r, hl = d_l < n_l;
    if (!hr && !hl) return false;
    const bool take_r = hr && (!hl || d_r * n_l <= d_l * n_r);
    TileCursor& c = take_r ? rc : lc;
    out = tile_of(c.locate(segs, nseg), c.t);
    c.t += gridDim.x;
    if (take_r) ++d_r; else ++d_l;
    return true;
  }
};

// Launch arguments every copy kernel takes. The vector-copy kernels use only the first four.
struct RunArgs {
  uint64_t wait_limit_ns;  // bound of every mbarrier wait (TMA kernels)
  uint32_t flags;          // RS_RUN_* bits (TMA kernels)
  uint32_t* status;        // kStatus* bits, OR-ed by the kernel
};

template <int BLOCK, int U, int MINB, bool STREAM = false>
__global__ void __launch_bounds__(BLOCK, MINB) rs_copy_kernel(const DevSeg* __restrict__ segs, int32_t nseg, uint64_t ntiles,
                                                               uint64_t nremote, RunArgs run) {
  (void)run;  // the vector-copy kernel has no waits that could fail
  Schedule sch;
  sch.init(segs, nseg, ntiles, nremote);
  Tile x;
  while (sch.next(segs, nseg, x)) {
    const uint32_t vpr = (uint32_t)(x.nb >> x.vshift);
    switch (x.vshift) {
      case 4: copy_rect16<U, STREAM>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      // Narrow widths only serve entries whose addresses or pitches are not 16-byte aligned
      // (odd shapes); one load in flight per thread keeps their register cost off the main path.
      case 3: copy_rect<8, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      case 2: copy_rect<4, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      case 1: copy_rect<2, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      default: copy_rect<1, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// TMA variant: bulk copies through a shared-memory ring.
// One warp per CTA. Lane 0 cuts the CTA's tiles into row chunks (16-byte aligned entries only),
// packs them into 16 KB stages, loads a stage with cp.async.bulk (global -> shared, completing
// on the stage's mbarrier) and writes it out with cp.async.bulk (shared -> global). LOOKAHEAD
// stages are in flight at once. Entries that are not 16-byte aligned are copied by the whole warp
// with vector loads. Every mbarrier wait is bounded by %globaltimer: past the limit the kernel
// sets kStatusWaitTimeout in *status, drains what it issued (bounded again) and stops.
// ---------------------------------------------------------------------------------------------
constexpr uint32_t kStatusWaitTimeout = 1u;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s, the default bound of every wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n selp.b32 %0, 1, 0, P;\n}"
      : "=r"(ok) : "r"(bar), "r"(phase) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase, uint64_t limit_ns) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, phase))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}
__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* gsrc, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_dst), "l"(gsrc), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int STAGES, int STAGE_BYTES, int MAXE>
struct TmaSmem {
  struct Ent {
    uint64_t src, dst;
    uint32_t off, bytes;
    uint64_t pad;
  };
  alignas(128) unsigned char buf[STAGES][STAGE_BYTES];
  Ent ent[STAGES][MAXE];
  uint64_t bar[STAGES];
  uint32_t count[STAGES];
  uint32_t bytes[STAGES];
};

template <int STAGES, int STAGE_BYTES, int MAXE, int LOOKAHEAD>
struct TmaPipe {
  using Smem = TmaSmem<STAGES, STAGE_BYTES, MAXE>;
  Smem& sm;
  uint32_t filled = 0;   // stages issued
  uint32_t retired = 0;  // stages stored
  bool failed = false;
  const RunArgs& run;

  __device__ TmaPipe(Smem& s, const RunArgs& r) : sm(s), run(r) {}

  __device__ uint32_t cur() const { return filled % STAGES; }

  // Chunk appended to the stage being filled; the stage is issued when full.
  __device__ void add(const char* src, char* dst, uint32_t bytes) {
    while (bytes > 0 && !failed) {
      const uint32_t s = cur();
      const uint32_t room = STAGE_BYTES - sm.bytes[s];
      const uint32_t take = bytes < room ? bytes : room;
      auto& e = sm.ent[s][sm.count[s]++];
      e.src = reinterpret_cast<uint64_t>(src);
      e.dst = reinterpret_cast<uint64_t>(dst);
      e.off = sm.bytes[s];
      e.bytes = take;
      sm.bytes[s] += take;
      src += take;
      dst += take;
      bytes -= take;
      if (sm.bytes[s] == STAGE_BYTES || sm.count[s] == MAXE) issue();
    }
  }

  __device__ void issue() {
    const uint32_t s = cur();
    if (sm.count[s] == 0) return;
    if (filled - retired == LOOKAHEAD) retire();
    if (failed) return;
    // the buffer of stage s was last stored STAGES - LOOKAHEAD retires ago
    bulk_wait_read<STAGES - LOOKAHEAD>();
    const uint32_t bar = smem_u32(&sm.bar[s]);
    mbar_arrive_expect_tx(bar, sm.bytes[s]);
    // RS_RUN_STALL_FIRST_STAGE (tests of the error path): the first stage's barrier expects bytes
    // that no copy delivers, so its bounded wait runs out. No load is in flight into that stage.
    const bool stall = (run.flags & RS_RUN_STALL_FIRST_STAGE) && filled == 0;
    const uint32_t base = smem_u32(&sm.buf[s][0]);
    for (uint32_t i = 0; i < sm.count[s] && !stall; ++i) {
      const auto& e = sm.ent[s][i];
      bulk_load(base + e.off, reinterpret_cast<const void*>(e.src), e.bytes, bar);
    }
    ++filled;
    const uint32_t n = cur();
    sm.count[n] = 0;
    sm.bytes[n] = 0;
  }

  __device__ void retire() {
    const uint32_t s = retired % STAGES;
    const uint32_t phase = (retired / STAGES) & 1u;
    if (!mbar_wait_bounded(smem_u32(&sm.bar[s]), phase, run.wait_limit_ns)) {
      atomicOr(run.status, kStatusWaitTimeout);
      failed = true;
      return;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const uint32_t base = smem_u32(&sm.buf[s][0]);
    for (uint32_t i = 0; i < sm.count[s]; ++i) {
      const auto& e = sm.ent[s][i];
      bulk_store(reinterpret_cast<void*>(e.dst), base + e.off, e.bytes);
    }
    bulk_commit();
    ++retired;
  }

  __device__ void finish() {
    if (!failed) issue();
    while (!failed && retired < filled) retire();
    if (failed) {  // drain the loads still in flight (bounded) before the CTA's shared memory goes away
      for (uint32_t q = retired + 1; q < filled; ++q)
        (void)mbar_wait_bounded(smem_u32(&sm.bar[q % STAGES]), (q / STAGES) & 1u, run.wait_limit_ns);
    }
    bulk_wait_all();
  }
};

template <int STAGES, int STAGE_BYTES, int MAXE, int LOOKAHEAD, int MINB>
__global__ void __launch_bounds__(32, MINB) rs_copy_tma_kernel(const DevSeg* __restrict__ segs, int32_t nseg, uint64_t ntiles,
                                                               uint64_t nremote, RunArgs run) {
  using Pipe = TmaPipe<STAGES, STAGE_BYTES, MAXE, LOOKAHEAD>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  auto& sm = *reinterpret_cast<typename Pipe::Smem*>(smem_raw);
  const bool leader = threadIdx.x == 0;
  if (leader) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&sm.bar[s]), 1);
      sm.count[s] = 0;
      sm.bytes[s] = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  Pipe pipe(sm, run);
  Schedule sch;
  sch.init(segs, nseg, ntiles, nremote);
  Tile x;
  while (sch.next(segs, nseg, x)) {
    if (x.vshift == 4) {
      if (leader && !pipe.failed)
        for (uint32_t r = 0; r < x.nr; ++r) pipe.add(x.src + r * x.sp, x.dst + r * x.dp, (uint32_t)x.nb);
      continue;
    }
    const uint32_t vpr = (uint32_t)(x.nb >> x.vshift);
    switch (x.vshift) {
      case 3: copy_rect<8, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      case 2: copy_rect<4, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      case 1: copy_rect<2, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
      default: copy_rect<1, 1>(x.src, x.dst, x.nr, vpr, x.sp, x.dp); break;
    }
  }
  if (leader) pipe.finish();
}

// ---------------------------------------------------------------------------------------------
// Tensor-map variant: TMA boxes through a shared-memory ring (SUIKA_RS_VARIANT 9-17).
// Every local, 16-byte aligned entry is described to the TMA unit as two tensors of 8-byte
// elements, its source and its target, each its rows with their own pitch; one
// cp.async.bulk.tensor.3d load moves a box (whole rows, or a 2 KB-wide strided tile) into a
// shared-memory stage, and one cp.async.bulk.tensor.3d store writes it to the target. The TMA
// unit clips boxes at the tensor edges, so ragged tiles need no code. One thread per CTA issues
// everything; STAGES - 1 loads stay in flight behind the store being issued. Entries that do not
// qualify (remote, or not 16-byte aligned) are left to the vector-copy kernel in the same run.
// Tensor maps never describe another GPU's memory here and no load uses cluster multicast.
// ---------------------------------------------------------------------------------------------
// The maps are 3-D: (x, chunk, row). A row that divides into n equal chunks of c bytes (16 | c,
// 256 <= c <= 2 KB, n <= 256) is seen as (c / 8, n, rows) and a box spans whole rows, or as many
// chunks of one row as a stage holds; any other row is (row_bytes / 8, 1, rows) with boxes of up
// to 2 KB across it. Box k of a row band starts at x = k * xstep, chunk = k * ystep.
struct alignas(64) TensorEntry {
  CUtensorMap src;      // map of the source rows (pitch = source pitch)
  CUtensorMap dst;      // map of the target rows (pitch = target pitch)
  uint64_t tile_begin;  // global index of this entry's first box
  uint32_t col_boxes;   // boxes across a row
  uint32_t xstep;       // x of box k = k * xstep (8-byte elements; even, so x * 8 stays 16-byte aligned)
  uint32_t ystep;       // chunk of box k = k * ystep
  uint32_t box_h;       // box height in rows
  uint32_t box_bytes;   // bytes a box load always delivers to shared memory (the whole box)
  // Entries that are column slices of the same source rows (the pieces of a TP grow) form a group
  // of consecutive entries with one geometry and one tile_begin; the group's boxes are numbered
  // row band by row band across its members, so CTAs that run at the same time read whole source
  // rows. Ungrouped entries are groups of one.
  uint32_t group;       // entries in this entry's group
  uint32_t member;      // this entry's place in its group
};
static_assert(sizeof(TensorEntry) == 320, "TensorEntry layout");

__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar) : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int32_t x, int32_t y, int32_t z, uint32_t smem_src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];"
               ::"l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_src) : "memory");
}
// The same with an L2 cache policy (evict-first: every byte is read once and written once).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_3d_hint(uint32_t smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                                 uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], "
      "[%5], %6;"
      ::"r"(smem_dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy) : "memory");
}
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* map, int32_t x, int32_t y, int32_t z, uint32_t smem_src,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%1, %2, %3}], [%4], %5;"
               ::"l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_src), "l"(policy) : "memory");
}
// The maps were written to global memory by a host copy before the launch; acquire them for the
// tensor-map proxy before their first use.
__device__ __forceinline__ void tensormap_acquire(const CUtensorMap* map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

struct TensorCursor {
  int32_t si;
  uint64_t next_begin;
  __device__ void init(const TensorEntry* __restrict__ ents, int32_t n, uint64_t t) {
    int32_t lo = 0, hi = n - 1;
    while (lo < hi) {
      const int32_t mid = (lo + hi + 1) >> 1;
      if (ents[mid].tile_begin <= t) lo = mid; else hi = mid - 1;
    }
    si = lo;
    next_begin = (si + 1 < n) ? ents[si + 1].tile_begin : ~0ull;
  }
  __device__ const TensorEntry& locate(const TensorEntry* __restrict__ ents, int32_t n, uint64_t t) {
    while (t >= next_begin) {
      ++si;
      next_begin = (si + 1 < n) ? ents[si + 1].tile_begin : ~0ull;
    }
    return ents[si];
  }
};

template <int STAGES, int STAGE_BYTES>
constexpr size_t tensor_smem_bytes() {
  return (size_t)STAGES * STAGE_BYTES + 1024 + (size_t)STAGES * (8 + 16);
}

template <int STAGES, int STAGE_BYTES, bool EVICT_FIRST>
__global__ void __launch_bounds__(32, 1) rs_copy_tensor_kernel(const TensorEntry* __restrict__ ents, int32_t nent, uint64_t ntiles,
                                                               RunArgs run) {
  extern __shared__ unsigned char smem_raw[];
  if (threadIdx.x != 0) return;
  struct Slot {
    const CUtensorMap* dst;
    int32_t x, y, z;
  };
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // stage buffers start 1 KB aligned
  unsigned char* gbase = smem_raw + (base - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (size_t)STAGES * STAGE_BYTES);
  Slot* slots = reinterpret_cast<Slot*>(bars + STAGES);
  for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&bars[s]), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");

  const uint64_t b = blockIdx.x, g = gridDim.x;
  const uint64_t n = ntiles > b ? (ntiles - b + g - 1) / g : 0;
  if (n == 0) return;
  TensorCursor cur;
  cur.init(ents, nent, b);
  int32_t acquired = -1;
  uint64_t issued = 0;
  const bool stall_first = (run.flags & RS_RUN_STALL_FIRST_STAGE) != 0;
  const uint64_t policy = EVICT_FIRST ? l2_evict_first_policy() : 0;
  auto issue = [&]() {
    const uint64_t t = b + issued * g;
    const TensorEntry& last = cur.locate(ents, nent, t);  // the last member of the group holding box t
    const int32_t first = cur.si - (int32_t)last.member;
    if (cur.si != acquired) {
      for (int32_t q = first; q <= cur.si; ++q) {
        tensormap_acquire(&ents[q].src);
        tensormap_acquire(&ents[q].dst);
      }
      acquired = cur.si;
    }
    const uint32_t cb_all = last.col_boxes;
    const uint32_t per_band = last.group * cb_all;
    const uint32_t lt = (uint32_t)(t - last.tile_begin);
    const uint32_t rb = lt / per_band, in_band = lt - rb * per_band;
    const uint32_t m = in_band / cb_all, cb = in_band - m * cb_all;
    const TensorEntry& e = ents[first + (int32_t)m];
    const uint32_t s = (uint32_t)(issued % STAGES);
    Slot& sl = slots[s];
    sl.dst = &e.dst;
    sl.x = (int32_t)(cb * e.xstep);
    sl.y = (int32_t)(cb * e.ystep);
    sl.z = (int32_t)(rb * e.box_h);
    const uint32_t bar = smem_u32(&bars[s]);
    mbar_arrive_expect_tx(bar, e.box_bytes);
    // RS_RUN_STALL_FIRST_STAGE (tests of the error path): the first box's barrier expects bytes
    // that no load delivers, so its bounded wait runs out; nothing is in flight into that stage.
    if (!(stall_first && issued == 0)) {
      if (EVICT_FIRST) tma_load_3d_hint(base + s * (uint32_t)STAGE_BYTES, &e.src, sl.x, sl.y, sl.z, bar, policy);
      else tma_load_3d(base + s * (uint32_t)STAGE_BYTES, &e.src, sl.x, sl.y, sl.z, bar);
    }
    ++issued;
  };
  const uint64_t prologue = n < (uint64_t)(STAGES - 1) ? n : (uint64_t)(STAGES - 1);
  while (issued < prologue) issue();
  uint64_t k = 0;
  bool failed = false;
  for (; k < n; ++k) {
    const uint32_t s = (uint32_t)(k % STAGES);
    if (!mbar_wait_bounded(smem_u32(&bars[s]), (uint32_t)(k / STAGES) & 1u, run.wait_limit_ns)) {
      failed = true;
      break;
    }
    if (EVICT_FIRST) tma_store_3d_hint(slots[s].dst, slots[s].x, slots[s].y, slots[s].z, base + s * (uint32_t)STAGE_BYTES, policy);
    else tma_store_3d(slots[s].dst, slots[s].x, slots[s].y, slots[s].z, base + s * (uint32_t)STAGE_BYTES);
    bulk_commit();
    if (issued < n) {
      // the new box goes into the stage of box k - 1, whose store must have read it out
      bulk_wait_read<1>();
      issue();
    }
  }
  if (failed) {
    atomicOr(run.status, kStatusWaitTimeout);
    // loads that may still be in flight into shared memory (at most STAGES - 1, one per stage)
    for (uint64_t q = k; q < issued; ++q)
      (void)mbar_wait_bounded(smem_u32(&bars[q % STAGES]), (uint32_t)(q / STAGES) & 1u, run.wait_limit_ns);
  }
  bulk_wait_all();
}

// Launch shapes. Vector-copy variants: (threads per CTA, 16-byte loads in flight per thread, CTAs
// per SM), each with 64 KB of loads in flight per SM; on cfg2b (1 x B200, 128 KB tiles) they span
// 5.83-6.00 TB/s. TMA variants: one warp per CTA, (stages, stage bytes, stages in flight, CTAs per
// SM). Unset, SUIKA_RS_VARIANT picks shape 8 or 2 per table (kAutoLocalVariant / kAutoRemoteVariant
// below); both are 256 x 8 with two CTAs per SM.
struct Variant {
  int block, unroll, min_blocks;
  size_t smem;
  void (*fn)(const DevSeg*, int32_t, uint64_t, uint64_t, RunArgs);
};
using TmaA = TmaSmem<8, 16384, 32>;
using TmaB = TmaSmem<6, 16384, 32>;
using TmaC = TmaSmem<12, 16384, 32>;
const Variant kVariants[] = {
    {512, 4, 2, 0, rs_copy_kernel<512, 4, 2>},
    {256, 8, 2, 0, rs_copy_kernel<256, 8, 2>},
    {1024, 4, 1, 0, rs_copy_kernel<1024, 4, 1>},
    {512, 8, 1, 0, rs_copy_kernel<512, 8, 1>},
    {32, 0, 1, sizeof(TmaA), rs_copy_tma_kernel<8, 16384, 32, 6, 1>},
    {32, 0, 2, sizeof(TmaB), rs_copy_tma_kernel<6, 16384, 32, 4, 2>},
    {32, 0, 1, sizeof(TmaC), rs_copy_tma_kernel<12, 16384, 32, 10, 1>},
    {256, 8, 2, 0, rs_copy_kernel<256, 8, 2, true>},  // 8: variant 2 with streaming cache hints
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);
// Tensor-map launch shapes (SUIKA_RS_VARIANT 9-17): (stages, stage bytes, evict-first hints); one warp per CTA, CTAs
// per SM as shared memory allows (1 for about 192 KB of stages, 2 for about 96 KB). `vector` is the
// launch shape of the entries the tensor-map kernel leaves out; `wide_only` keeps it to the rows it
// reads fastest (wide_desc), leaving the narrower ones to the banded vector copy.
struct TensorShape {
  int stages, stage_bytes;
  size_t smem;
  void (*fn)(const TensorEntry*, int32_t, uint64_t, RunArgs);
  int vector;
  bool wide_only;
};
const TensorShape kTensorShapes[] = {
    {8, 24576, tensor_smem_bytes<8, 24576>(), rs_copy_tensor_kernel<8, 24576, false>, 1, false},
    {4, 24576, tensor_smem_bytes<4, 24576>(), rs_copy_tensor_kernel<4, 24576, false>, 1, false},
    {4, 49152, tensor_smem_bytes<4, 49152>(), rs_copy_tensor_kernel<4, 49152, false>, 1, false},
    {6, 16384, tensor_smem_bytes<6, 16384>(), rs_copy_tensor_kernel<6, 16384, false>, 1, false},
    {8, 24576, tensor_smem_bytes<8, 24576>(), rs_copy_tensor_kernel<8, 24576, true>, 1, false},  // 13: 9 with evict-first L2 hints
    {4, 49152, tensor_smem_bytes<4, 49152>(), rs_copy_tensor_kernel<4, 49152, true>, 1, false},  // 14: 11 with evict-first L2 hints
    {4, 49152, tensor_smem_bytes<4, 49152>(), rs_copy_tensor_kernel<4, 49152, false>, 7, true},  // 15: 11 for wide rows, 8 for the rest
    {4, 57344, tensor_smem_bytes<4, 57344>(), rs_copy_tensor_kernel<4, 57344, false>, 7, true},  // 16: 15 with 56 KB stages
    {3, 73728, tensor_smem_bytes<3, 73728>(), rs_copy_tensor_kernel<3, 73728, false>, 7, true},  // 17: 15 with 3 x 72 KB stages
};
static_assert(tensor_smem_bytes<4, 57344>() <= 232448 && tensor_smem_bytes<3, 73728>() <= 232448,
              "a tensor-map shape exceeds 227 KB of shared memory per CTA");
constexpr int kNumTensorShapes = sizeof(kTensorShapes) / sizeof(kTensorShapes[0]);

// Workspace layout: the staged vector-copy table, a 256-byte status block (word 0: kStatus* bits),
// then, for the tensor-map shapes, the TensorEntry table.
constexpr uint64_t kStatusBytes = 256;
constexpr uint64_t kBandEntriesPerDesc = 16;  // workspace room per descriptor, in vector-copy entries
uint64_t status_offset(int64_t n_entries) { return ((uint64_t)n_entries * sizeof(DevSeg) + 255) & ~255ull; }
uint64_t tensor_offset(int64_t n_entries) { return status_offset(n_entries) + kStatusBytes; }

uint64_t env_u64(const char* name, uint64_t dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  char* end = nullptr;
  const unsigned long long x = std::strtoull(v, &end, 10);
  return (end && *end == 0 && x > 0) ? (uint64_t)x : dflt;
}

// Launch shape chosen by SUIKA_RS_VARIANT (1-based): 0-based index below kNumVariants for the
// vector and bulk-copy kernels, kNumVariants + i for tensor-map shape i. Unset (or 0) selects per
// table: a table whose entries all stay in this GPU's memory runs shape 17 (wide rows and long
// runs through the tensor-map kernel with 3 x 72 KB stages, the other rows through the vector
// shape 8 with evict-first stores and band-interleaved TP-grow slices: the fastest split on a
// one-GPU relayout); a table
// with any entry that crosses NVLink, or reads host memory, runs the vector shape 2, whose CTAs
// interleave remote and local tiles so both links stay busy.
constexpr int kAutoVariant = -1;
constexpr int kAutoLocalVariant = kNumVariants + 8;  // tensor-map shape 17 (SUIKA_RS_VARIANT=17)
constexpr int kAutoRemoteVariant = 1;
static_assert(kAutoLocalVariant == 16 && kAutoLocalVariant < kNumVariants + kNumTensorShapes,
              "the one-GPU default must be a tensor-map shape");
int selected_variant() {
  const uint64_t v = env_u64("SUIKA_RS_VARIANT", 0);
  if (v == 0) return kAutoVariant;
  return (int)std::min<uint64_t>(v - 1, kNumVariants + kNumTensorShapes - 1);
}
bool is_tensor_variant(int v) { return v >= kNumVariants; }
// Launch shape of the vector-copy part of a run.
int vector_variant_of(int v) { return is_tensor_variant(v) ? kTensorShapes[v - kNumVariants].vector : v; }

// Rows the tensor-map kernel reads faster than the banded vector copy (one-GPU probe of column
// slices of 4096-row matrices): half-rows wider than 8 KB, and contiguous runs of 1 MB or more.
// Narrower half-rows (8 KB, 4 KB) go faster through the vector copy's row bands.
bool wide_desc(const rs_copy_desc& d) {
  const bool contiguous = d.rows == 1 || (d.src_pitch == d.row_bytes && d.dst_pitch == d.row_bytes);
  return contiguous ? d.rows * d.row_bytes >= (1ull << 20) : d.row_bytes > 8192;
}

// cuTensorMapEncodeTiled, looked up once through the runtime (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
int encode_tiled_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      return efail(RS_ERR_CUDA, "rs_copy_stage: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return RS_OK;
}

// Largest power of two <= 16 dividing every address, pitch and row length of the entry.
uint32_t vector_shift(const rs_copy_desc& d) {
  const uint64_t bits = d.src_dev | d.dst_dev | d.row_bytes | (d.rows > 1 ? (d.src_pitch | d.dst_pitch) : 0);
  uint32_t s = 4;
  while (s > 0 && (bits & ((1ull << s) - 1))) --s;
  return s;
}

// One descriptor -> one table entry (validated), its tiles numbered from `ntiles`.
int make_entry(const rs_copy_desc& d, int64_t i, uint64_t tile_bytes, uint64_t& ntiles, DevSeg& s, const char* fn) {
  if (d.rows > 0xffffffffull) return efail(RS_ERR_ARG, std::string(fn) + ": entry " + std::to_string(i) + " has more than 2^32 rows");
  if (d.rows > 1 && (d.row_bytes > d.src_pitch || d.row_bytes > d.dst_pitch))
    return efail(RS_ERR_ARG, std::string(fn) + ": entry " + std::to_string(i) + " has rows longer than their pitch");
  if (!d.src_dev || !d.dst_dev) return efail(RS_ERR_ARG, std::string(fn) + ": entry " + std::to_string(i) + " has a NULL address");
  s.src = d.src_dev;
  s.dst = d.dst_dev;
  s.src_pitch = d.src_pitch;
  s.dst_pitch = d.dst_pitch;
  s.rows = (uint32_t)d.rows;
  s.row_bytes = d.row_bytes;
  s.vshift = vector_shift(d);
  s.tile_begin = ntiles;
  if (d.row_bytes >= tile_bytes) {
    s.col_bytes = tile_bytes;
    s.col_tiles = (uint32_t)((d.row_bytes + tile_bytes - 1) / tile_bytes);
    s.rows_per_tile = 1;
    ntiles += (uint64_t)s.col_tiles * d.rows;
  } else {
    s.col_bytes = d.row_bytes;
    s.col_tiles = 1;
    // Whole rows per tile, capped so that every in-tile offset fits 32 bits.
    const uint64_t pitch = std::max(d.src_pitch, d.dst_pitch);
    const uint64_t rows_32 = pitch ? (0xffffffffull - d.row_bytes) / pitch + 1 : 1;
    s.rows_per_tile = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(tile_bytes / d.row_bytes, rows_32));
    ntiles += (d.rows + s.rows_per_tile - 1) / s.rows_per_tile;
  }
  return RS_OK;
}

bool empty_desc(const rs_copy_desc& d) { return d.rows == 0 || d.row_bytes == 0; }
bool remote_desc(const rs_copy_desc& d) { return (d.flags & RS_COPY_REMOTE) != 0; }

struct IndexedDesc {
  rs_copy_desc d;
  int64_t index;  // position in the caller's table, for error messages
};

// Column slices of the same source rows (the pieces of a TP grow: one source row split between
// several targets) are read at different times when each slice is its own entry: the first
// slice's tiles all come before the second's. DRAM then serves each source row twice, half a row
// at a time, and a one-GPU relayout stays 5 % below a plain copy. Here such slices are cut into
// row bands of about `band_bytes` per slice and the bands of a group are interleaved (band 0 of
// every slice, then band 1, ...), so the CTAs that run at the same time read whole source rows.
// Bands are kept large (8 MB by default, about 64 tiles) because a CTA steps over the entries
// between its tiles one by one. band_bytes = 0 keeps the table as it is.
// At most max_out entries come out: a group whose bands would not fit gets fewer, taller bands,
// or stays whole.
constexpr uint64_t kDefaultBandBytes = 8ull << 20;
std::vector<IndexedDesc> band_interleave(const std::vector<IndexedDesc>& in, uint64_t band_bytes, uint64_t max_out) {
  if (band_bytes == 0 || in.size() < 2 || max_out <= in.size()) return in;
  uint64_t budget = max_out - in.size();  // entries the cuts may add
  const size_t n = in.size();
  std::vector<size_t> idx;
  for (size_t i = 0; i < n; ++i)
    if (in[i].d.rows > 1) idx.push_back(i);
  std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
    const rs_copy_desc &x = in[a].d, &y = in[b].d;
    if (x.src_pitch != y.src_pitch) return x.src_pitch < y.src_pitch;
    if (x.rows != y.rows) return x.rows < y.rows;
    if (x.row_bytes != y.row_bytes) return x.row_bytes < y.row_bytes;
    return x.src_dev < y.src_dev;
  });
  std::vector<char> grouped(n, 0);
  std::vector<IndexedDesc> groups_out;
  for (size_t i = 0; i < idx.size();) {
    const rs_copy_desc& d0 = in[idx[i]].d;
    size_t j = i + 1;
    while (j < idx.size() && j - i < 8) {
      const rs_copy_desc& dj = in[idx[j]].d;
      const rs_copy_desc& dp = in[idx[j - 1]].d;
      const bool same = dj.src_pitch == d0.src_pitch && dj.rows == d0.rows && dj.row_bytes == d0.row_bytes;
      if (!same || dj.src_dev - d0.src_dev >= d0.src_pitch || dj.src_dev - dp.src_dev < dp.row_bytes) break;
      ++j;
    }
    const uint64_t k = j - i;
    uint64_t band_rows = std::max<uint64_t>(1, band_bytes / d0.row_bytes);
    uint64_t bands = (d0.rows + band_rows - 1) / band_rows;
    if (k >= 2 && bands > 1 && k * (bands - 1) > budget) {  // not enough room: fewer, taller bands
      bands = 1 + budget / k;
      band_rows = (d0.rows + bands - 1) / bands;
      bands = (d0.rows + band_rows - 1) / band_rows;
    }
    if (k >= 2 && bands > 1) {
      budget -= k * (bands - 1);
      for (uint64_t r0 = 0; r0 < d0.rows; r0 += band_rows) {
        const uint64_t nr = std::min(band_rows, d0.rows - r0);
        for (size_t q = i; q < j; ++q) {
          IndexedDesc x = in[idx[q]];
          x.d.src_dev += r0 * x.d.src_pitch;
          x.d.dst_dev += r0 * x.d.dst_pitch;
          x.d.rows = nr;
          groups_out.push_back(x);
        }
      }
      for (size_t q = i; q < j; ++q) grouped[idx[q]] = 1;
    }
    i = j;
  }
  std::vector<IndexedDesc> out;
  out.reserve(n + groups_out.size());
  for (size_t i = 0; i < n; ++i)
    if (!grouped[i]) out.push_back(in[i]);
  out.insert(out.end(), groups_out.begin(), groups_out.end());
  return out;
}

// An entry the tensor-map kernel takes: this GPU's memory on both sides, 16-byte aligned addresses
// and pitches (the TMA rules for a tensor's base and strides), whole 8-byte elements per row.
bool tensor_desc(const rs_copy_desc& d) {
  if (remote_desc(d) || (d.src_dev | d.dst_dev) & 15 || d.row_bytes & 7) return false;
  if (d.rows > 1 && ((d.src_pitch | d.dst_pitch) & 15)) return false;
  return d.rows < (1ull << 31) && d.row_bytes / 8 <= (1ull << 32);
}

// A 3-D map of 8-byte elements: dims (x, chunk, row), strides in bytes (chunk, row).
int encode_3d(EncodeTiledFn fn, CUtensorMap* m, uint64_t addr, const uint64_t dim[3], uint64_t chunk_stride, uint64_t pitch,
              const uint32_t box[3]) {
  const cuuint64_t dims[3] = {dim[0], dim[1], dim[2]};
  const cuuint64_t strides[2] = {chunk_stride, pitch};
  const cuuint32_t boxd[3] = {box[0], box[1], box[2]};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, reinterpret_cast<void*>(addr), dims, strides, boxd, elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return efail(RS_ERR_CUDA, "rs_copy_stage: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return RS_OK;
}

// Host-side geometry of a TensorEntry (the maps themselves are opaque).
struct TensorGeom {
  uint64_t src, src_pitch, rows, row_bytes;
};

// One rows x row_bytes rectangle -> one TensorEntry, its boxes numbered from `ntiles`. A row that
// splits into equal chunks (see TensorEntry) gets boxes of whole rows, as many as a stage holds,
// so loads read and stores write whole rows; a row longer than a stage gets boxes of as many of
// its chunks as fit. Any other row gets boxes 2 KB wide (a narrower row: one box as wide as the
// row, rounded up to an even element count) and as tall as the stage holds.
int add_tensor_entry(EncodeTiledFn fn, uint64_t src, uint64_t dst, uint64_t rows, uint64_t row_bytes, uint64_t sp, uint64_t dp,
                     uint32_t stage_bytes, uint64_t& ntiles, std::vector<TensorEntry>& out, std::vector<TensorGeom>& geom) {
  const uint64_t cols = row_bytes / 8;
  if (rows == 1) sp = dp = (row_bytes + 15) & ~15ull;  // one row: the stride only has to be legal
  uint64_t chunk = 0;  // whole-row boxes: the widest chunk c dividing the row with 16 | c and n <= 256
  for (uint64_t c = std::min<uint64_t>(2048, row_bytes) & ~15ull; c >= 256; c -= 16)
    if (row_bytes % c == 0 && row_bytes / c <= 256) {
      chunk = c;
      break;
    }
  uint64_t dim[3];
  uint32_t box[3];
  uint64_t chunk_stride;
  TensorEntry te;
  std::memset(&te, 0, sizeof(te));
  if (chunk) {
    const uint64_t n = row_bytes / chunk;
    const uint64_t bn = row_bytes <= stage_bytes ? n : std::max<uint64_t>(1, stage_bytes / chunk);
    const uint64_t bh = row_bytes <= stage_bytes ? std::min<uint64_t>(std::min<uint64_t>(rows, 256), stage_bytes / row_bytes) : 1;
    dim[0] = chunk / 8; dim[1] = n; dim[2] = rows;
    box[0] = (uint32_t)(chunk / 8); box[1] = (uint32_t)bn; box[2] = (uint32_t)bh;
    chunk_stride = chunk;
    te.col_boxes = (uint32_t)((n + bn - 1) / bn);
    te.xstep = 0;
    te.ystep = (uint32_t)bn;
  } else {  // boxes of up to 2 KB across the row (an even element count, so x stays 16-byte aligned)
    uint64_t bw = std::min<uint64_t>(cols, 256);
    bw += bw & 1;
    const uint64_t bh = std::min<uint64_t>(std::min<uint64_t>(rows, 256), std::max<uint64_t>(1, stage_bytes / (bw * 8)));
    dim[0] = cols; dim[1] = 1; dim[2] = rows;
    box[0] = (uint32_t)bw; box[1] = 1; box[2] = (uint32_t)bh;
    chunk_stride = (row_bytes + 15) & ~15ull;
    te.col_boxes = (uint32_t)((cols + bw - 1) / bw);
    te.xstep = (uint32_t)bw;
    te.ystep = 0;
  }
  te.box_h = box[2];
  te.box_bytes = box[0] * 8 * box[1] * box[2];
  te.tile_begin = ntiles;
  te.group = 1;
  te.member = 0;
  int rc = encode_3d(fn, &te.src, src, dim, chunk_stride, sp, box);
  if (!rc) rc = encode_3d(fn, &te.dst, dst, dim, chunk_stride, dp, box);
  if (rc) return rc;
  ntiles += (uint64_t)te.col_boxes * ((rows + te.box_h - 1) / te.box_h);
  out.push_back(te);
  geom.push_back(TensorGeom{src, sp, rows, row_bytes});
  return RS_OK;
}

// A descriptor -> tensor entries. A contiguous run (one row, or pitches equal to the row) is seen
// as 2 KB rows plus a shorter last row, so its boxes are full-width.
int make_tensor_entries(EncodeTiledFn fn, const rs_copy_desc& d, uint32_t stage_bytes, uint64_t& ntiles,
                        std::vector<TensorEntry>& out, std::vector<TensorGeom>& geom) {
  const bool contiguous = d.rows == 1 || (d.src_pitch == d.row_bytes && d.dst_pitch == d.row_bytes);
  const uint64_t total = d.rows * d.row_bytes;
  if (contiguous && total >= 4096) {
    const uint64_t w = 2048, main_rows = total / w, rem = total % w;
    int rc = add_tensor_entry(fn, d.src_dev, d.dst_dev, main_rows, w, w, w, stage_bytes, ntiles, out, geom);
    if (!rc && rem)
      rc = add_tensor_entry(fn, d.src_dev + main_rows * w, d.dst_dev + main_rows * w, 1, rem, rem, rem, stage_bytes, ntiles, out, geom);
    return rc;
  }
  return add_tensor_entry(fn, d.src_dev, d.dst_dev, d.rows, d.row_bytes, d.src_pitch, d.dst_pitch, stage_bytes, ntiles, out, geom);
}

// Reorder the tensor entries so that column slices of the same source rows sit together as
// groups (at most 8: a TP grow by up to 8), and renumber the boxes from `first_tile`. Two entries
// join when they have the same rows, row length and source pitch, and their sources lie within one
// source row of each other without overlapping. Returns the total number of boxes.
uint64_t group_tensor_entries(std::vector<TensorEntry>& ents, const std::vector<TensorGeom>& geom, uint64_t first_tile) {
  const size_t n = ents.size();
  std::vector<size_t> idx(n);
  for (size_t i = 0; i < n; ++i) idx[i] = i;
  std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
    const TensorGeom &x = geom[a], &y = geom[b];
    if (x.src_pitch != y.src_pitch) return x.src_pitch < y.src_pitch;
    if (x.rows != y.rows) return x.rows < y.rows;
    if (x.row_bytes != y.row_bytes) return x.row_bytes < y.row_bytes;
    return x.src < y.src;
  });
  std::vector<TensorEntry> out;
  out.reserve(n);
  uint64_t tile = first_tile;
  for (size_t i = 0; i < n;) {
    const TensorGeom& g0 = geom[idx[i]];
    size_t j = i + 1;
    while (j < n && j - i < 8 && g0.rows > 1) {
      const TensorGeom& gj = geom[idx[j]];
      const TensorGeom& gp = geom[idx[j - 1]];
      const bool same = gj.src_pitch == g0.src_pitch && gj.rows == g0.rows && gj.row_bytes == g0.row_bytes;
      if (!same || gj.src - g0.src >= g0.src_pitch || gj.src - gp.src < gp.row_bytes) break;
      ++j;
    }
    const TensorEntry& lead = ents[idx[i]];
    const uint64_t boxes = (uint64_t)lead.col_boxes * ((g0.rows + lead.box_h - 1) / lead.box_h);
    for (size_t q = i; q < j; ++q) {
      TensorEntry e = ents[idx[q]];
      e.tile_begin = tile;
      e.group = (uint32_t)(j - i);
      e.member = (uint32_t)(q - i);
      out.push_back(e);
    }
    tile += boxes * (j - i);
    i = j;
  }
  ents.swap(out);
  return tile - first_tile;
}

}  // namespace

extern "C" {

int rs_copy_workspace_bytes(int64_t n_desc, uint64_t* bytes) {
  if (!bytes || n_desc < 0) return efail(RS_ERR_ARG, "rs_copy_workspace_bytes: bad argument");
  // room for the row-band cuts of the vector copy (up to kBandEntriesPerDesc entries per descriptor)
  *bytes = (((uint64_t)n_desc * kBandEntriesPerDesc * sizeof(DevSeg) + 255) & ~255ull) + kStatusBytes;
  const int v = selected_variant();
  if (v == kAutoVariant || is_tensor_variant(v)) *bytes += 2 * (uint64_t)n_desc * sizeof(TensorEntry);  // a run may become 2 entries
  return RS_OK;
}

int rs_copy_stage(const rs_copy_desc* descs, int64_t n_desc, void* workspace_dev, uint64_t workspace_bytes, void* stream,
                  rs_launch_info* info) {
  if (!info) return efail(RS_ERR_ARG, "rs_copy_stage: info is NULL");
  std::memset(info, 0, sizeof(*info));
  if (n_desc < 0 || (n_desc > 0 && !descs)) return efail(RS_ERR_ARG, "rs_copy_stage: bad descriptor array");
  const uint64_t tile_bytes = std::min<uint64_t>(1ull << 30, std::max<uint64_t>(256, env_u64("SUIKA_RS_TILE_BYTES", kDefaultTileBytes))) & ~15ull;
  int variant = selected_variant();
  if (variant == kAutoVariant) {
    bool any_remote = false;
    for (int64_t i = 0; i < n_desc && !any_remote; ++i) any_remote = !empty_desc(descs[i]) && remote_desc(descs[i]);
    variant = any_remote ? kAutoRemoteVariant : kAutoLocalVariant;
  }
  const bool tensor = is_tensor_variant(variant);
  EncodeTiledFn encode = nullptr;  // looked up at the first tensor entry, after its validation
  std::vector<DevSeg> table;
  std::vector<TensorEntry> tensor_table;
  std::vector<TensorGeom> tensor_geom;
  std::vector<IndexedDesc> local_vec;  // local entries of the vector copy, placed after the loop
  table.reserve((size_t)n_desc);
  uint64_t ntiles = 0, total = 0, nremote = 0, ntensor_tiles = 0;
  for (int pass = 0; pass < 2; ++pass) {  // remote entries first, then local ones
    for (int64_t i = 0; i < n_desc; ++i) {
      const rs_copy_desc& d = descs[i];
      if (empty_desc(d) || remote_desc(d) != (pass == 0)) continue;
      DevSeg sg;
      int rc = make_entry(d, i, tile_bytes, ntiles, sg, "rs_copy_stage");  // validates the descriptor either way
      if (rc) return rc;
      total += d.rows * d.row_bytes;
      if (tensor && tensor_desc(d) && (!kTensorShapes[variant - kNumVariants].wide_only || wide_desc(d))) {
        ntiles = sg.tile_begin;  // not a vector-copy entry after all
        if (!encode && (rc = encode_tiled_fn(&encode))) return rc;
        rc = make_tensor_entries(encode, d, (uint32_t)kTensorShapes[variant - kNumVariants].stage_bytes, ntensor_tiles, tensor_table,
                                 tensor_geom);
        if (rc) return rc;
        continue;
      }
      if (pass == 0) {
        table.push_back(sg);
      } else {
        ntiles = sg.tile_begin;
        local_vec.push_back(IndexedDesc{d, i});
      }
    }
    if (pass == 0) nremote = ntiles;
  }
  // entries the caller's workspace holds besides the status block and the tensor maps
  const uint64_t tensor_room = tensor ? 2 * (uint64_t)n_desc * sizeof(TensorEntry) : 0;
  const uint64_t room = workspace_bytes > kStatusBytes + tensor_room + 256 ? (workspace_bytes - kStatusBytes - tensor_room - 256) / sizeof(DevSeg) : 0;
  const uint64_t max_local = std::min<uint64_t>((uint64_t)n_desc * kBandEntriesPerDesc, room > table.size() ? room - table.size() : 0);
  for (const IndexedDesc& x : band_interleave(local_vec, env_u64("SUIKA_RS_BAND_BYTES", kDefaultBandBytes), max_local)) {
    DevSeg sg;
    const int rc = make_entry(x.d, x.index, tile_bytes, ntiles, sg, "rs_copy_stage");
    if (rc) return rc;
    table.push_back(sg);
  }
  if (!tensor_table.empty()) ntensor_tiles = group_tensor_entries(tensor_table, tensor_geom, 0);
  info->n_entries = (int64_t)table.size();
  info->n_tiles = ntiles;
  info->n_tiles_remote = nremote;
  info->total_bytes = total;
  info->variant = variant;
  info->n_tensor_entries = (int64_t)tensor_table.size();
  info->n_tensor_tiles = ntensor_tiles;
  if (table.empty() && tensor_table.empty()) return RS_OK;
  if (table.size() > 0x7fffffffull || tensor_table.size() > 0x7fffffffull) return efail(RS_ERR_ARG, "rs_copy_stage: too many entries");
  const uint64_t need = tensor_offset((int64_t)table.size()) + tensor_table.size() * sizeof(TensorEntry);
  if (!workspace_dev || workspace_bytes < need)
    return efail(RS_ERR_CAPACITY, "rs_copy_stage: workspace of " + std::to_string(workspace_bytes) + " bytes, need " + std::to_string(need));
  if (reinterpret_cast<uintptr_t>(workspace_dev) & 255) return efail(RS_ERR_ARG, "rs_copy_stage: workspace must be 256-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Pageable source: the runtime copies the table out before returning, so it may be freed.
  cudaError_t e = cudaSuccess;
  if (!table.empty()) {
    e = cudaMemcpyAsync(workspace_dev, table.data(), table.size() * sizeof(DevSeg), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_stage: staging the copy table");
  }
  if (!tensor_table.empty()) {
    e = cudaMemcpyAsync(static_cast<char*>(workspace_dev) + tensor_offset((int64_t)table.size()), tensor_table.data(),
                        tensor_table.size() * sizeof(TensorEntry), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_stage: staging the tensor maps");
  }
  e = cudaMemsetAsync(static_cast<char*>(workspace_dev) + status_offset((int64_t)table.size()), 0, kStatusBytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "rs_copy_stage: clearing the status block");
  int dev = 0, sms = 0, per_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  const uint64_t cap_per_sm = env_u64("SUIKA_RS_CTAS_PER_SM", 8);
  const Variant& v = kVariants[vector_variant_of(variant)];
  if (!table.empty()) {
    if (v.smem > 0 &&
        (e = cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v.smem)) != cudaSuccess)
      return cuda_fail(e, "rs_copy_stage: cudaFuncSetAttribute");
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v.fn, v.block, v.smem)) != cudaSuccess)
      return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    per_sm = (int)std::min<uint64_t>((uint64_t)std::max(per_sm, 1), cap_per_sm);
    info->grid = (int32_t)std::min<uint64_t>(ntiles, (uint64_t)sms * (uint64_t)per_sm);
    info->block = v.block;
  }
  if (!tensor_table.empty()) {
    const TensorShape& ts = kTensorShapes[variant - kNumVariants];
    if ((e = cudaFuncSetAttribute(ts.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ts.smem)) != cudaSuccess)
      return cuda_fail(e, "rs_copy_stage: cudaFuncSetAttribute (tensor-map kernel)");
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ts.fn, 32, ts.smem)) != cudaSuccess)
      return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    per_sm = (int)std::min<uint64_t>((uint64_t)std::max(per_sm, 1), cap_per_sm);
    info->tensor_grid = (int32_t)std::min<uint64_t>(ntensor_tiles, (uint64_t)sms * (uint64_t)per_sm);
    info->tensor_block = 32;
  }
  return RS_OK;
}

int rs_copy_run_bounded(const void* workspace_dev, const rs_launch_info* info, void* stream, uint64_t wait_limit_ns,
                        uint32_t flags) {
  if (!info) return efail(RS_ERR_ARG, "rs_copy_run: info is NULL");
  const bool vec_part = info->n_entries > 0 && info->n_tiles > 0;
  const bool tensor_part = info->n_tensor_entries > 0 && info->n_tensor_tiles > 0;
  if (!vec_part && !tensor_part) return RS_OK;
  if (!workspace_dev || info->variant < 0 || info->variant >= kNumVariants + kNumTensorShapes || (vec_part && info->grid <= 0) ||
      (tensor_part && (info->tensor_grid <= 0 || !is_tensor_variant(info->variant))))
    return efail(RS_ERR_ARG, "rs_copy_run: info does not come from rs_copy_stage");
  if (wait_limit_ns == 0) return efail(RS_ERR_ARG, "rs_copy_run_bounded: the wait limit must be positive");
  if (flags & ~(uint32_t)RS_RUN_STALL_FIRST_STAGE) return efail(RS_ERR_ARG, "rs_copy_run_bounded: unknown flag bits");
  const bool tensor = is_tensor_variant(info->variant);
  const Variant& v = kVariants[vector_variant_of(info->variant)];
  if ((flags & RS_RUN_STALL_FIRST_STAGE) && !(tensor ? tensor_part : v.smem > 0))
    return efail(RS_ERR_ARG, "rs_copy_run_bounded: RS_RUN_STALL_FIRST_STAGE needs a TMA launch shape (SUIKA_RS_VARIANT 5-7 or 9-17)");
  char* ws = static_cast<char*>(const_cast<void*>(workspace_dev));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  RunArgs run;
  run.wait_limit_ns = wait_limit_ns;
  run.flags = flags;
  run.status = reinterpret_cast<uint32_t*>(ws + status_offset(info->n_entries));
  if (vec_part) {
    RunArgs vrun = run;
    if (tensor) vrun.flags = 0;  // the stall hook is meant for the tensor-map kernel
    v.fn<<<(unsigned)info->grid, v.block, v.smem, st>>>(reinterpret_cast<const DevSeg*>(ws), (int32_t)info->n_entries, info->n_tiles,
                                                        info->n_tiles_remote, vrun);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_run: kernel launch");
  }
  if (tensor_part) {
    const TensorShape& ts = kTensorShapes[info->variant - kNumVariants];
    ts.fn<<<(unsigned)info->tensor_grid, 32, ts.smem, st>>>(reinterpret_cast<const TensorEntry*>(ws + tensor_offset(info->n_entries)),
                                                           (int32_t)info->n_tensor_entries, info->n_tensor_tiles, run);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_run: tensor-map kernel launch");
  }
  return RS_OK;
}

int rs_copy_run(const void* workspace_dev, const rs_launch_info* info, void* stream) {
  return rs_copy_run_bounded(workspace_dev, info, stream, kWaitLimitNs, 0);
}

int rs_copy_status(const void* workspace_dev, const rs_launch_info* info, void* stream, uint32_t* status) {
  if (!info || !status) return efail(RS_ERR_ARG, "rs_copy_status: NULL argument");
  *status = 0;
  if (info->n_entries == 0 && info->n_tensor_entries == 0) return RS_OK;
  if (!workspace_dev) return efail(RS_ERR_ARG, "rs_copy_status: NULL workspace");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, static_cast<const char*>(workspace_dev) + status_offset(info->n_entries), sizeof(v),
                                  cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "rs_copy_status: reading the status block");
  *status = v;
  return RS_OK;
}

int rs_copy_launch(const rs_copy_desc* descs, int64_t n_desc, void* workspace_dev, uint64_t workspace_bytes, void* stream,
                   rs_launch_info* info) {
  rs_launch_info local;
  rs_launch_info* li = info ? info : &local;
  int rc = rs_copy_stage(descs, n_desc, workspace_dev, workspace_bytes, stream, li);
  if (rc) return rc;
  return rs_copy_run(workspace_dev, li, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Peer memory: CUDA IPC export/import of the allocations that hold source tensors. A target
// rank maps each peer allocation it reads once and pulls from it with rs_copy_launch.
// ---------------------------------------------------------------------------------------------
namespace {
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int address_range(const void* ptr, uint64_t* base, uint64_t* bytes) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return efail(RS_ERR_PEER, "rs_peer_export: cuMemGetAddressRange entry point unavailable");
  CUdeviceptr b = 0;
  size_t n = 0;
  const CUresult r = reinterpret_cast<GetAddressRangeFn>(fn)(&b, &n, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return efail(RS_ERR_PEER, "rs_peer_export: cuMemGetAddressRange failed (" + std::to_string((int)r) + ")");
  *base = (uint64_t)b;
  *bytes = (uint64_t)n;
  return RS_OK;
}
}  // namespace

extern "C" {

int rs_host_device_pointer(const void* host_ptr, void** dev_ptr) {
  if (!host_ptr || !dev_ptr) return efail(RS_ERR_ARG, "rs_host_device_pointer: NULL argument");
  *dev_ptr = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(dev_ptr, const_cast<void*>(host_ptr), 0);
  if (e != cudaSuccess) return cuda_fail(e, "rs_host_device_pointer: cudaHostGetDevicePointer (memory must be page-locked)");
  return RS_OK;
}

int rs_peer_export(const void* ptr_dev, rs_peer_handle* out, uint64_t* offset) {
  if (!ptr_dev || !out || !offset) return efail(RS_ERR_ARG, "rs_peer_export: NULL argument");
  std::memset(out, 0, sizeof(*out));
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr_dev);
  if (e != cudaSuccess) return cuda_fail(e, "rs_peer_export: cudaPointerGetAttributes");
  if (attr.type != cudaMemoryTypeDevice) return efail(RS_ERR_PEER, "rs_peer_export: pointer is not device memory");
  uint64_t base = 0, bytes = 0;
  int rc = address_range(ptr_dev, &base, &bytes);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base))) != cudaSuccess)
    return cuda_fail(e, "rs_peer_export: cudaIpcGetMemHandle (the allocation must come from cudaMalloc; "
                        "PyTorch's expandable segments are not exportable this way)");
  static_assert(sizeof(h) <= sizeof(out->ipc), "IPC handle size");
  std::memcpy(out->ipc, &h, sizeof(h));
  out->alloc_base = base;
  out->alloc_bytes = bytes;
  out->device = attr.device;
  out->pid = (int32_t)getpid();
  *offset = (uint64_t)reinterpret_cast<uintptr_t>(ptr_dev) - base;
  return RS_OK;
}

int rs_peer_open(const rs_peer_handle* handle, void** base_dev) {
  if (!handle || !base_dev) return efail(RS_ERR_ARG, "rs_peer_open: NULL argument");
  *base_dev = nullptr;
  if (handle->pid == (int32_t)getpid())
    return efail(RS_ERR_PEER, "rs_peer_open: handle exported by this process; use the local address");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->ipc, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "rs_peer_open: cudaIpcOpenMemHandle");
  *base_dev = p;
  return RS_OK;
}

int rs_peer_close(void* base_dev) {
  if (!base_dev) return efail(RS_ERR_ARG, "rs_peer_close: NULL argument");
  cudaError_t e = cudaIpcCloseMemHandle(base_dev);
  if (e != cudaSuccess) return cuda_fail(e, "rs_peer_close: cudaIpcCloseMemHandle");
  return RS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Copy launch that allocates nothing (rs_copy_launch_noalloc). Its copy table lives in a
// file-scope device array instead of caller-provided workspace.
// ---------------------------------------------------------------------------------------------
namespace {

// Every GPU that loads this library holds this array (RS_NOALLOC_MAX_ENTRIES x 72 bytes, about
// 1.2 MB) until the process exits. All calls share it.
static __device__ __align__(256) DevSeg g_noalloc_table[RS_NOALLOC_MAX_ENTRIES];

constexpr int kMaxDevices = 64;
// Device address of g_noalloc_table per device ordinal, set once by the first call on that device.
DevSeg* g_noalloc_addr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

int noalloc_table_addr(int dev, DevSeg** out) {
  if (dev < 0 || dev >= kMaxDevices) return efail(RS_ERR_ARG, "rs_copy_launch_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    // In host code the array's name is only a stand-in; the device address has to be looked up,
    // with the device current.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_table);
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_launch_noalloc: cudaGetSymbolAddress");
    g_noalloc_addr[dev] = static_cast<DevSeg*>(p);
  }
  *out = g_noalloc_addr[dev];
  return RS_OK;
}

// The no-allocation launch runs only the vector-copy kernels: they have no waits, so there is no
// status a caller would have to read back. Unset, or set to a TMA variant, SUIKA_RS_VARIANT gives
// the vector shape 2 here.
int noalloc_variant() {
  const int v = selected_variant();
  return (v != kAutoVariant && !is_tensor_variant(v) && kVariants[v].smem == 0) ? v : 1;
}

}  // namespace

extern "C" {

int rs_copy_launch_noalloc(const rs_copy_desc* descs, int64_t n_desc, void* stream, rs_launch_info* info) {
  rs_launch_info local;
  rs_launch_info* li = info ? info : &local;
  std::memset(li, 0, sizeof(*li));
  if (n_desc < 0 || (n_desc > 0 && !descs)) return efail(RS_ERR_ARG, "rs_copy_launch_noalloc: bad descriptor array");
  int64_t n_entries = 0;
  for (int64_t i = 0; i < n_desc; ++i)
    if (!empty_desc(descs[i])) ++n_entries;
  if (n_entries > RS_NOALLOC_MAX_ENTRIES)
    return efail(RS_ERR_CAPACITY, "rs_copy_launch_noalloc: " + std::to_string(n_entries) + " non-empty copies, at most " +
                                      std::to_string(RS_NOALLOC_MAX_ENTRIES) + " fit the built-in table; use rs_copy_launch");
  if (n_entries == 0) return RS_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DevSeg* table = nullptr;
  int rc = noalloc_table_addr(dev, &table);
  if (rc) return rc;
  const uint64_t tile_bytes = std::min<uint64_t>(1ull << 30, std::max<uint64_t>(256, env_u64("SUIKA_RS_TILE_BYTES", kDefaultTileBytes))) & ~15ull;
  const int variant = noalloc_variant();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Stage in chunks through a stack buffer: no heap memory on the host either. Pageable copies
  // are taken out of the buffer before cudaMemcpyAsync returns, so the buffer can be refilled.
  constexpr int kChunk = 128;
  DevSeg chunk[kChunk];
  int nc = 0;
  int64_t written = 0;
  uint64_t ntiles = 0, total = 0;
  uint64_t nremote = 0;
  for (int pass = 0; pass < 2; ++pass) {  // remote entries first, then local ones
    for (int64_t i = 0; i < n_desc; ++i) {
      const rs_copy_desc& d = descs[i];
      if (empty_desc(d) || remote_desc(d) != (pass == 0)) continue;
      if (written + nc >= n_entries) return efail(RS_ERR_ARG, "rs_copy_launch_noalloc: descriptor count changed while staging");
      rc = make_entry(d, i, tile_bytes, ntiles, chunk[nc++], "rs_copy_launch_noalloc");
      if (rc) return rc;
      total += d.rows * d.row_bytes;
      if (nc == kChunk) {
        e = cudaMemcpyAsync(table + written, chunk, nc * sizeof(DevSeg), cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "rs_copy_launch_noalloc: staging the copy table");
        written += nc;
        nc = 0;
      }
    }
    if (pass == 0) nremote = ntiles;
  }
  if (nc > 0) {
    e = cudaMemcpyAsync(table + written, chunk, nc * sizeof(DevSeg), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "rs_copy_launch_noalloc: staging the copy table");
    written += nc;
  }
  if (written != n_entries) return efail(RS_ERR_ARG, "rs_copy_launch_noalloc: staged entry count differs from the count");
  int sms = 0, per_sm = 0;
  const Variant& v = kVariants[variant];
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v.fn, v.block, v.smem)) != cudaSuccess)
    return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  per_sm = (int)std::min<uint64_t>((uint64_t)std::max(per_sm, 1), env_u64("SUIKA_RS_CTAS_PER_SM", 8));
  li->n_entries = n_entries;
  li->n_tiles = ntiles;
  li->n_tiles_remote = nremote;
  li->total_bytes = total;
  li->variant = variant;
  li->grid = (int32_t)std::min<uint64_t>(ntiles, (uint64_t)sms * (uint64_t)per_sm);
  li->block = v.block;
  // The vector-copy kernels have no waits and never write a status word.
  RunArgs run;
  run.wait_limit_ns = kWaitLimitNs;
  run.flags = 0;
  run.status = nullptr;
  v.fn<<<(unsigned)li->grid, v.block, 0, st>>>(table, (int32_t)n_entries, ntiles, nremote, run);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "rs_copy_launch_noalloc: kernel launch");
  return RS_OK;
}

}  // extern "C"
