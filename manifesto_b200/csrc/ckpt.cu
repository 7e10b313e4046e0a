// ckpt.cu -- the checkpoint quantisation step in one launch (mf_ckpt_plan_*).
//
// Per-tensor amax scaling is a global dependency: no element of a tensor can be
// cast before every element of it has been seen.  The two-pass form
// (mf_ckpt_quant_fp8) therefore reads every source byte twice from DRAM:
// 2 + 2 + 1 = 5 bytes per BF16 parameter.  This form cuts the tensors into
// groups of consecutive tensors (32 MB of this rank's source by default) and
// runs one persistent kernel.  Its schedule is a sequence of segments;
// segment k interleaves, tile by tile, the amax tiles of group k (read from
// DRAM with an evict-last L2 policy) with the cast tiles of group k - 1 (read
// again, evict-first, while they are still in the 126 MB L2), so the DRAM
// reads of one group overlap the cast arithmetic of the previous one and DRAM
// traffic falls towards the single-pass bound of 3 bytes per BF16 parameter
// (read once, write FP8 once).  A tensor too large for the L2 budget is cast
// from DRAM again, as in the two-pass form.
//
// Every CTA gets a contiguous range of each group's tiles; the CTAs that take
// the group's one extra tile start after the group's first tile number, so the
// extra tile moves from CTA to CTA from group to group (MF_PLAN_DEAL=1 deals
// tiles round-robin instead, measured slower).
//
// The cast tiles of a group need its amax over every CTA and every rank.  When
// a CTA has folded its amax tiles of group g its consumer warps meet at a named
// barrier and one thread arrives on the group's counter.  One GPU: a CTA
// about to cast group g waits (acquire, bounded) for the counter to reach the
// grid size.  Several: the last CTA to arrive publishes the group's per-tensor
// maxima into a slot of every rank's exchange buffer (plain stores over NVLink
// into peer memory opened with CUDA IPC; no multicast) and then sets, on every
// rank, a per-group flag to the run's epoch with a system-scope release; a CTA
// about to cast group g waits for every rank's flag and takes the maximum over
// the slots.  Each segment opens with a few amax tiles before its first cast
// tile, which gives the last CTAs of the previous segment time to arrive.
//
// Safety: the launch is cooperative (every CTA resident, so a CTA that waits
// never waits on a CTA that cannot run); every wait is bounded (mbarriers by
// poll count, groups by 2 s of %globaltimer).  A group wait that runs out marks
// the run abandoned: later waits of the run return at once and skip their cast
// work, amax tiles are still folded and published (so other ranks are not held
// up), and the host reads MF_DEVICE_TIMEOUT from the sticky status.  A warp
// whose bulk-copy stage never lands skips its remaining tile work but keeps
// every barrier and arrival.
//
// Double buffering by epoch parity: slots and per-run scratch (local amax,
// arrival counters, the abandon word) come in two copies; a run uses copy
// epoch & 1 and clears the other for the next run.  A peer can be at most one
// run ahead in its amax work (its cast work waits on this rank's flags), so it
// only ever writes the copy this rank is not reading; flags are compared as
// "at least this epoch".
#include <algorithm>
#include <cstring>
#include <vector>

#include "mf_internal.h"
#include "mf_runtime.h"
#include "mf_stream.cuh"

namespace mf {
namespace {

// Compile-time tunables (the defaults are the measured choices):
//   MF_PLAN_LEAD        amax tiles that open a segment before its first cast tile
//   MF_PLAN_STAGE_KB    shared-memory staging per CTA (tiles of 16384 16-bit or 8192 32-bit elements)
//   MF_PLAN_CTAS        CTAs per SM
//   MF_PLAN_AMAX_HINT   L2 policy of the amax phase's loads (0 none, 1 evict_last, 2 evict_first)
//   MF_PLAN_CAST_HINT   L2 policy of the cast phase's loads
//   MF_PLAN_REVERSE     1: the cast phase walks each CTA's tiles last to first (the tiles the amax
//                       phase read last are the likeliest still in L2)
//   MF_PLAN_DEAL        1: tiles dealt round-robin across CTAs; 0: contiguous ranges
//   MF_PLAN_GROUP_MB    default group budget
#ifndef MF_PLAN_LEAD
#define MF_PLAN_LEAD 8
#endif
#ifndef MF_PLAN_STAGE_KB
#define MF_PLAN_STAGE_KB 64
#endif
#ifndef MF_PLAN_CTAS
#define MF_PLAN_CTAS 2
#endif
#ifndef MF_PLAN_AMAX_HINT
#define MF_PLAN_AMAX_HINT 1
#endif
#ifndef MF_PLAN_CAST_HINT
#define MF_PLAN_CAST_HINT 2
#endif
#ifndef MF_PLAN_REVERSE
#define MF_PLAN_REVERSE 0
#endif
#ifndef MF_PLAN_DEAL
#define MF_PLAN_DEAL 0
#endif
#ifndef MF_PLAN_GROUP_MB
#define MF_PLAN_GROUP_MB 32
#endif

constexpr int64_t kPlanLead = MF_PLAN_LEAD;
constexpr int kPlanCtas = MF_PLAN_CTAS;
constexpr int64_t kDefaultGroupBytes = int64_t(MF_PLAN_GROUP_MB) << 20;

struct PlanGroup {
    int32_t t0, t1;  // tensors [t0, t1)
    int32_t c0, c1;  // chunks [c0, c1) of the plan's chunk table (tile_begin relative to the group)
    int64_t tiles;
    int64_t base;    // tiles of the groups before this one (the round-robin deal continues from there)
};

struct PlanArgs {
    const ChunkRec* chunks;
    const PlanGroup* groups;
    float* local_amax;   // [2][n_tensors]   this GPU's amax of its own chunks
    int32_t* arrivals;   // [2][n_groups]    warps that finished a group's amax phase
    int32_t* abandon;    // [2]              set when a flag wait ran out
    float* out_amax;     // [n_tensors] global amax, or NULL
    float* out_scale_inv;
    int* status;
    float* slots[kPlanMaxWorld];    // rank p's slots: [2][world][n_tensors]
    int32_t* flags[kPlanMaxWorld];  // rank p's flags: [n_groups][world]
    int32_t n_groups, n_tensors, world, rank, epoch, pad;
};

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 1-D bulk copy global -> shared with an L2 eviction policy (no multicast).
__device__ __forceinline__ void bulk_g2s_policy(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// a tile's bulk copy with the L2 policy code HINT (0 none, 1 evict_last, 2 evict_first)
template <int HINT>
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t last, uint64_t first) {
    if constexpr (HINT == 1) bulk_g2s_policy(dst, src, bytes, bar, last);
    else if constexpr (HINT == 2) bulk_g2s_policy(dst, src, bytes, bar, first);
    else bulk_g2s(dst, src, bytes, bar);
}


// ------------------------------------------------------- amax of a tile

// Running magnitude key of a lane, monotone in |v| and never NaN.  16-bit
// formats: one max.xorsign.abs per word keeps max(|a|, |b|) per half (the
// maxNum rule: a NaN half never wins; the sign bits are the XOR of the inputs'
// and mean nothing -- key_to_f32 clears them).  float32: (bits & 0x7fffffff)
// of non-NaN values.
template <int SRC>
__device__ __forceinline__ uint32_t fold_word(uint32_t key, uint32_t w) {
    if constexpr (SRC == MF_DT_F32) {
        const uint32_t a = w & 0x7fffffffu;
        return (a <= 0x7f800000u && a > key) ? a : key;
    } else if constexpr (SRC == MF_DT_BF16) {
        uint32_t r;
        asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(key), "r"(w));
        return r;
    } else {
        uint32_t r;
        asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(key), "r"(w));
        return r;
    }
}
template <int SRC>
__device__ __forceinline__ float key_to_f32(uint32_t key) {
    if constexpr (SRC == MF_DT_F32) {
        return __uint_as_float(key);
    } else {
        const uint32_t h = max(key & 0x7fffu, (key >> 16) & 0x7fffu);
        if constexpr (SRC == MF_DT_BF16) return __uint_as_float(h << 16);
        else return __uint_as_float(f16_to_f32bits(h));
    }
}
template <int SRC>
__device__ __forceinline__ float abs_elem(const void* p, int64_t i) {
    const float a = fabsf(load_as_f32<SRC>(p, i));
    return (a == a) ? a : 0.0f;
}

// ---------------------------------------------------------------- kernel

template <class Op>
struct PlanGeometry {
    static constexpr int64_t kTileElems = stream_tile_elems<Op::kIn>();
    static constexpr int kTileBytes = static_cast<int>(kTileElems) * Op::kIn;
    static constexpr int kStages = (MF_PLAN_STAGE_KB * 1024 / kTileBytes) < 8 ? (MF_PLAN_STAGE_KB * 1024 / kTileBytes) : 8;
    static constexpr int kFixOffset = kStages * kTileBytes + kStages * 16;
    static constexpr int kFixBytes = Op::kDefers ? kConsumerWarps * kFixSlots * (32 + 8) : 0;
    static constexpr int kSmemBytes = kFixOffset + kFixBytes;
    static_assert(kStages >= 2, "tile too large for the staging budget");
};

// This CTA's tiles of a group.  Tiles are dealt round-robin over one numbering
// that continues across groups (tile base + t goes to CTA (base + t) mod grid):
// within a group CTAs differ by at most one tile, and the CTA that gets the
// extra one moves on from group to group, so no CTA falls behind over a run.
struct CtaTiles {
    int64_t first, count, step;
    __device__ __forceinline__ int64_t tile(int64_t j, bool reverse) const {
        return first + (reverse ? count - 1 - j : j) * step;
    }
};
__device__ __forceinline__ CtaTiles cta_tiles(const PlanGroup& grp) {
    const int64_t n = gridDim.x;
#if MF_PLAN_DEAL
    int64_t f = (static_cast<int64_t>(blockIdx.x) - grp.base) % n;
    if (f < 0) f += n;
    return {f, grp.tiles > f ? (grp.tiles - 1 - f) / n + 1 : 0, n};
#else
    // contiguous ranges, the extra tiles going to the CTAs after this group's base
    const int64_t per = grp.tiles / n, extra = grp.tiles % n;
    int64_t b = (static_cast<int64_t>(blockIdx.x) - grp.base) % n;
    if (b < 0) b += n;
    const int64_t lo = b * per + (b < extra ? b : extra);
    return {lo, per + (b < extra ? 1 : 0), 1};
#endif
}

// The chunk of [c0, c1) that holds group tile t.
__device__ __forceinline__ int group_chunk(const ChunkRec* ch, int c0, int c1, int64_t t) {
    int lo = c0, hi = c1 - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ch[mid].tile_begin <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// The chunk of the tile last asked for, with its tile range [lo, hi) in the
// group: a CTA's tiles of a group come in order, so the chunk table is searched
// only when a tile leaves the current chunk.
struct ChunkCursor {
    int k = 0;
    int64_t lo = 0, hi = -1;
    __device__ __forceinline__ void reset() { lo = 0; hi = -1; }
    __device__ __forceinline__ const ChunkRec& at(const ChunkRec* ch, const PlanGroup& g, int64_t t) {
        if (t < lo || t >= hi) {
            k = group_chunk(ch, g.c0, g.c1, t);
            lo = ch[k].tile_begin;
            hi = (k + 1 < g.c1) ? ch[k + 1].tile_begin : g.tiles;
        }
        return ch[k];
    }
};

// Warp 0 of the CTA: wait until group g's amax is complete on every rank (one GPU:
// every CTA of this launch has arrived; several: every rank has published).
// Returns false when the wait ran out or the run was abandoned.
__device__ bool wait_group(const PlanArgs& a, int g, const int32_t* arrivals, int32_t* abandon) {
    const int lane = threadIdx.x & 31;
    bool ok = ld_relaxed_gpu(abandon) == 0;
    if (ok && lane < a.world) {
        const unsigned long long t0 = globaltimer_ns();
        if (a.world == 1) {
            const int32_t* c = arrivals + g;
            int32_t v;
            for (;;) {
                asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
                if (v >= static_cast<int32_t>(gridDim.x)) break;
                if (globaltimer_ns() - t0 > kFlagWaitNs || ld_relaxed_gpu(abandon) != 0) {
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        } else {
            // flags only grow; "at least this epoch" (a peer may already be one run ahead)
            const int32_t* f = a.flags[a.rank] + static_cast<int64_t>(g) * a.world + lane;
            while (static_cast<int32_t>(static_cast<uint32_t>(ld_acquire_sys(f)) - static_cast<uint32_t>(a.epoch)) < 0) {
                if (globaltimer_ns() - t0 > kFlagWaitNs || ld_relaxed_gpu(abandon) != 0) {
                    ok = false;
                    break;
                }
                __nanosleep(128);
            }
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) {
        atomicExch(abandon, 1);
        atomicExch(a.status, kDeviceTimeout);
    }
    return ok;
}

// Global amax of tensor t once its group is complete (warp-collective): one GPU
// reads the local maximum; several take the max over the ranks' slots.
__device__ __forceinline__ float global_amax(const PlanArgs& a, int par, const float* lam, int t) {
    if (a.world == 1) return ld_relaxed_gpu(lam + t);
    const int lane = threadIdx.x & 31;
    float v = 0.0f;
    if (lane < a.world)
        v = ld_relaxed_sys(a.slots[a.rank] + (static_cast<int64_t>(par) * a.world + lane) * a.n_tensors + t);
    return warp_max_f32(v);
}

// Warp-collective, by warp 0 of the last CTA to finish group g's amax phase on
// this GPU (several ranks only): this GPU's per-tensor maxima into every
// rank's slot, then the flags.
__device__ void publish_group(const PlanArgs& a, const PlanGroup& grp, int g, int par, const float* lam) {
    const int lane = threadIdx.x & 31;
    for (int p = 0; p < a.world; ++p) {
        float* dst = a.slots[p] + (static_cast<int64_t>(par) * a.world + a.rank) * a.n_tensors;
        for (int t = grp.t0 + lane; t < grp.t1; t += 32) dst[t] = ld_relaxed_gpu(lam + t);
    }
    __threadfence_system();
    __syncwarp();
    if (lane < a.world) st_release_sys(a.flags[lane] + static_cast<int64_t>(g) * a.world + a.rank, a.epoch);
}

// One segment of a CTA's schedule: segment k holds this CTA's amax tiles of
// group k (na) and its cast tiles of group k - 1 (nc), interleaved so that the
// DRAM reads of the amax tiles overlap the arithmetic of the cast tiles (which
// read their data from L2).  The segment opens with kPlanLead amax tiles
// (slack for the last CTAs to finish group k - 1 before the first cast tile
// needs it), and the remaining amax tiles are spread over the first three
// quarters of the cast tiles, so the CTA's part of group k is done well before
// the segment ends.  Producer and consumers walk the same order.
struct Segment {
    int64_t na, nc, ia = 0, ic = 0;
    __device__ __forceinline__ bool next_is_amax() const {
        if (ia >= na) return false;
        if (ic >= nc || ia < kPlanLead) return true;
        const int64_t lead = kPlanLead;
        return (ia - lead) * nc * 3 <= ic * (na - lead) * 4;
    }
    __device__ __forceinline__ bool done() const { return ia >= na && ic >= nc; }
};

template <int SRC, int FP8, int COMPAT>
__global__ void __launch_bounds__(kStreamBlock, kPlanCtas) ckpt_plan_kernel(const __grid_constant__ PlanArgs a) {
    using Op = CastOp<SRC, FP8, COMPAT>;
    using G = PlanGeometry<Op>;
    constexpr int kIn = Op::kIn;
    constexpr bool kRev = MF_PLAN_REVERSE != 0;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kTileBytes);
    uint64_t* empty = full + G::kStages;
    __shared__ int s_leader;    // this CTA arrived last on a group (several ranks: it publishes)
    __shared__ int s_ready[4];  // a group is complete (slot g & 3)
    const int par = a.epoch & 1;
    const int n_groups = a.n_groups;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (threadIdx.x >= kStreamThreads) {
        // ------------- producer: one lane streams every tile of the schedule
        if (threadIdx.x != kStreamThreads) return;
        const uint64_t keep = l2_policy_evict_last(), drop = l2_policy_evict_first();
        int64_t i = 0;
        bool ok = true;
        ChunkCursor cur_a, cur_c;
        for (int k = 0; k <= n_groups && ok; ++k) {
            cur_a.reset();
            cur_c.reset();
            PlanGroup ga{}, gc{};
            CtaTiles ta{0, 0, 1}, tc{0, 0, 1};
            if (k < n_groups) {
                ga = a.groups[k];
                ta = cta_tiles(ga);
            }
            if (k >= 1) {
                gc = a.groups[k - 1];
                tc = cta_tiles(gc);
            }
            Segment sg{ta.count, tc.count};
            while (!sg.done()) {
                const bool am = sg.next_is_amax();
                const PlanGroup& grp = am ? ga : gc;
                const int64_t t = am ? ta.tile(sg.ia++, false) : tc.tile(sg.ic++, kRev);
                const int st = static_cast<int>(i % G::kStages);
                if (i >= G::kStages && !mbar_wait(&empty[st], static_cast<uint32_t>((i / G::kStages - 1) & 1))) {
                    ok = false;
                    break;
                }
                ++i;
                const ChunkRec& ch = am ? cur_a.at(a.chunks, grp, t) : cur_c.at(a.chunks, grp, t);
                const int64_t e0 = (t - ch.tile_begin) * G::kTileElems;
                const int64_t cnt = min(G::kTileElems, ch.n - e0);
                const uint32_t bytes = static_cast<uint32_t>((cnt * kIn) & ~int64_t(15));
                if (ch.aligned && bytes > 0) {
                    mbar_arrive_expect_tx(&full[st], bytes);
                    void* sd = smem + st * G::kTileBytes;
                    const void* gs = static_cast<const uint8_t*>(ch.src) + e0 * kIn;
                    if (am) bulk_g2s_hint<MF_PLAN_AMAX_HINT>(sd, gs, bytes, &full[st], keep, drop);
                    else bulk_g2s_hint<MF_PLAN_CAST_HINT>(sd, gs, bytes, &full[st], keep, drop);
                } else {
                    mbar_arrive(&full[st]);
                }
            }
        }
        if (!ok) atomicExch(a.status, kDeviceTimeout);
        for (int64_t j = (i > G::kStages ? i - G::kStages : 0); j < i; ++j)
            mbar_wait(&full[j % G::kStages], static_cast<uint32_t>((j / G::kStages) & 1));
        return;
    }

    // ------------------------------------------ consumers (warps 0..7)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* lam = a.local_amax + static_cast<int64_t>(par) * a.n_tensors;
    int32_t* arrivals = a.arrivals + static_cast<int64_t>(par) * n_groups;
    int32_t* abandon = a.abandon + par;
    if (blockIdx.x == 0) {
        // clear the other copy of the per-run scratch for the next run (the
        // previous run, its last user, has finished: runs are stream-ordered)
        const int nx = par ^ 1;
        for (int t = threadIdx.x; t < a.n_tensors; t += kStreamThreads) a.local_amax[int64_t(nx) * a.n_tensors + t] = 0.0f;
        for (int g = threadIdx.x; g < n_groups; g += kStreamThreads) a.arrivals[int64_t(nx) * n_groups + g] = 0;
        if (threadIdx.x == 0) a.abandon[nx] = 0;
    }
    FixQueue fq;
    fq.v = reinterpret_cast<float4*>(smem + G::kFixOffset) + warp * 2 * kFixSlots;
    fq.d = reinterpret_cast<uint8_t**>(smem + G::kFixOffset + kConsumerWarps * kFixSlots * 32) + warp * kFixSlots;
    fq.n = 0;
    fq.age = 0;

    // A warp whose stage never landed (a bounded mbarrier wait ran out) skips all
    // remaining tile work, but still takes part in every barrier of the CTA and
    // every arrival, so no other warp, CTA or rank waits on it for ever.
    bool dead = false;
    int64_t i = 0;

    // the CTA's part of group g's amax is done: flush, one arrival, publish if last
    auto finish_amax = [&](int g, const PlanGroup& grp, int cur, uint32_t key, float mel) {
        if (cur >= 0) {
            const float m = warp_max_f32(fmaxf(key_to_f32<SRC>(key), mel));
            if (lane == 0 && m > 0.0f) atomicMax(reinterpret_cast<unsigned*>(lam + cur), __float_as_uint(m));
        }
        consumers_sync();
        if (threadIdx.x == 0) {
            __threadfence();
            const int old = atomicAdd(arrivals + g, 1);
            s_leader = (a.world > 1 && old == static_cast<int>(gridDim.x) - 1) ? 1 : 0;
        }
        consumers_sync();
        if (s_leader && warp == 0) {
            __threadfence();
            publish_group(a, grp, g, par, lam);
        }
    };
    // wait for group g to be complete everywhere; the group's writer CTA also
    // stores its amax / scale_inv outputs.  CTA-collective; returns readiness.
    auto wait_cast = [&](int g, const PlanGroup& grp, bool writer) -> bool {
        if (warp == 0) {
            const bool ok = wait_group(a, g, arrivals, abandon);
            if (lane == 0) s_ready[g & 3] = ok ? 1 : 0;
            if (ok && writer) {
                for (int t = grp.t0; t < grp.t1; ++t) {
                    const float ga = global_amax(a, par, lam, t);
                    if (lane == 0) {
                        if (a.out_amax) a.out_amax[t] = ga;
                        if (a.out_scale_inv) a.out_scale_inv[t] = scale_inv_from_amax(ga, FP8);
                    }
                }
            }
        }
        consumers_sync();
        return s_ready[g & 3] != 0;
    };

    for (int k = 0; k <= n_groups; ++k) {
        PlanGroup ga{}, gc{};
        CtaTiles ta{0, 0, 1}, tc{0, 0, 1};
        if (k < n_groups) {
            ga = a.groups[k];
            ta = cta_tiles(ga);
        }
        if (k >= 1) {
            gc = a.groups[k - 1];
            tc = cta_tiles(gc);
        }
        const bool writer = k >= 1 && static_cast<int>(blockIdx.x) == (k - 1) % static_cast<int>(gridDim.x);
        Segment sg{ta.count, tc.count};
        ChunkCursor ccur_a, ccur_c;
        uint32_t key = 0;
        float mel = 0.0f;
        int cur_a = -1, cur_c = -1;
        typename Op::State stt{1.0f};
        bool waited = false, ready = false;
        while (!sg.done()) {
            const bool am = sg.next_is_amax();
            if (!am && !waited) {
                ready = wait_cast(k - 1, gc, writer);
                waited = true;
            }
            const PlanGroup& grp = am ? ga : gc;
            const int64_t t = am ? ta.tile(sg.ia++, false) : tc.tile(sg.ic++, kRev);
            const int st = static_cast<int>(i % G::kStages);
            const uint32_t phase = static_cast<uint32_t>((i / G::kStages) & 1);
            ++i;
            if (!dead && !__all_sync(0xffffffffu, mbar_wait(&full[st], phase))) {
                if (lane == 0) atomicExch(a.status, kDeviceTimeout);
                dead = true;
            }
            if (!dead) {
                const ChunkRec& ch = am ? ccur_a.at(a.chunks, grp, t) : ccur_c.at(a.chunks, grp, t);
                const int64_t e0 = (t - ch.tile_begin) * G::kTileElems;
                const int64_t cnt = min(G::kTileElems, ch.n - e0);
                if (am) {
                    // ---- amax tile: fold max|v| of the tensor
                    if (ch.tensor != cur_a) {
                        if (cur_a >= 0) {
                            const float m = warp_max_f32(fmaxf(key_to_f32<SRC>(key), mel));
                            if (lane == 0 && m > 0.0f) atomicMax(reinterpret_cast<unsigned*>(lam + cur_a), __float_as_uint(m));
                        }
                        cur_a = ch.tensor;
                        key = 0;
                        mel = 0.0f;
                    }
                    if (ch.aligned) {
                        const int64_t copied = ((cnt * kIn) & ~int64_t(15));
                        const uint4* tp = reinterpret_cast<const uint4*>(smem + st * G::kTileBytes);
                        if (cnt == G::kTileElems) {
                            constexpr int kVecs = G::kTileBytes / 16 / kStreamThreads;
#pragma unroll
                            for (int v = 0; v < kVecs; ++v) {
                                const uint4 w = tp[threadIdx.x + v * kStreamThreads];
                                key = fold_word<SRC>(fold_word<SRC>(fold_word<SRC>(fold_word<SRC>(key, w.x), w.y), w.z), w.w);
                            }
                        } else {
                            for (int v = threadIdx.x; v < copied / 16; v += kStreamThreads) {
                                const uint4 w = tp[v];
                                key = fold_word<SRC>(fold_word<SRC>(fold_word<SRC>(fold_word<SRC>(key, w.x), w.y), w.z), w.w);
                            }
                            for (int64_t e = e0 + copied / kIn + threadIdx.x; e < e0 + cnt; e += kStreamThreads)
                                mel = fmaxf(mel, abs_elem<SRC>(ch.src, e));
                        }
                    } else {
                        for (int64_t e = e0 + threadIdx.x; e < e0 + cnt; e += kStreamThreads)
                            mel = fmaxf(mel, abs_elem<SRC>(ch.src, e));
                    }
                } else if (ready) {
                    // ---- cast tile: scale by the tensor's global amax, encode, store
                    if (ch.tensor != cur_c) {
                        cur_c = ch.tensor;
                        stt.scale = scale_from_amax(global_amax(a, par, lam, cur_c), FP8);
                    }
                    if (ch.aligned) {
                        const uint8_t* tp = smem + st * G::kTileBytes;
                        if (cnt == G::kTileElems) {
                            constexpr int kStepsPerThread = static_cast<int>(G::kTileElems / Op::kLane / kStreamThreads);
#pragma unroll
                            for (int q0 = 0; q0 < kStepsPerThread; ++q0) {
                                const int q = threadIdx.x + q0 * kStreamThreads;
                                Op::template step<Op::kDefers>(tp + q * Op::kLane * kIn, ch, e0 + Op::kLane * q, stt, fq);
                            }
                            if constexpr (Op::kDefers)
                                if (fq.n && (fq.n >= kDrainSlots || ++fq.age >= kDrainTiles)) fix_drain<Op>(fq);
                        } else {
                            const int copied = static_cast<int>(((cnt * kIn) & ~int64_t(15)) / kIn);
                            const int nsteps = copied / Op::kLane;
                            for (int q = threadIdx.x; q < nsteps; q += kStreamThreads)
                                Op::template step<false>(tp + q * Op::kLane * kIn, ch, e0 + Op::kLane * q, stt, fq);
                            const int rem = static_cast<int>(cnt) - nsteps * Op::kLane;
                            if (threadIdx.x < rem) Op::element(ch, e0 + nsteps * Op::kLane + threadIdx.x, stt);
                        }
                    } else {
                        for (int64_t e = e0 + threadIdx.x; e < e0 + cnt; e += kStreamThreads) Op::element(ch, e, stt);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
            if (am && sg.ia == sg.na) finish_amax(k, ga, cur_a, key, mel);
        }
        if (k < n_groups && sg.na == 0) finish_amax(k, ga, -1, 0u, 0.0f);  // no tiles of group k: arrive all the same
        if (k >= 1 && !waited && writer) wait_cast(k - 1, gc, true);
    }
    if constexpr (Op::kDefers)
        if (fq.n) fix_drain<Op>(fq);
}

using PlanKernel = void (*)(PlanArgs);

template <int SRC, int FP8>
PlanKernel pick_compat(int compat) {
    return compat ? ckpt_plan_kernel<SRC, FP8, 1> : ckpt_plan_kernel<SRC, FP8, 0>;
}
template <int SRC>
PlanKernel pick_fp8(int fp8, int compat) {
    return fp8 == MF_DT_F8E4M3 ? pick_compat<SRC, MF_DT_F8E4M3>(compat) : pick_compat<SRC, MF_DT_F8E5M2>(compat);
}
PlanKernel pick_kernel(int src, int fp8, int compat, int* smem_bytes, int64_t* tile_elems) {
    switch (src) {
    case MF_DT_F32:
        *smem_bytes = PlanGeometry<CastOp<MF_DT_F32, MF_DT_F8E4M3, 0>>::kSmemBytes;
        *tile_elems = stream_tile_elems<4>();
        return pick_fp8<MF_DT_F32>(fp8, compat);
    case MF_DT_F16:
        *smem_bytes = PlanGeometry<CastOp<MF_DT_F16, MF_DT_F8E4M3, 0>>::kSmemBytes;
        *tile_elems = stream_tile_elems<2>();
        return pick_fp8<MF_DT_F16>(fp8, compat);
    default:
        *smem_bytes = PlanGeometry<CastOp<MF_DT_BF16, MF_DT_F8E4M3, 0>>::kSmemBytes;
        *tile_elems = stream_tile_elems<2>();
        return pick_fp8<MF_DT_BF16>(fp8, compat);
    }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace mf

struct mf_ckpt_plan_s {
    int device = -1;
    int world = 1, rank = 0, n_tensors = 0, n_groups = 0;
    int src_dtype = MF_DT_BF16, fp8 = MF_DT_F8E4M3, compat = 0;
    int grid = 0, smem_bytes = 0;
    int64_t total_tiles = 0, elems = 0;
    mf::PlanKernel kernel = nullptr;
    mf::ChunkRec* d_chunks = nullptr;
    mf::PlanGroup* d_groups = nullptr;
    uint8_t* d_scratch = nullptr;  // local amax [2][T] | arrivals [2][G] | abandon [2], counter [2]
    size_t arrivals_off = 0, abandon_off = 0, counter_off = 0;
    uint8_t* d_xbuf = nullptr;     // flags [G][world] | slots [2][world][T]
    size_t slots_off = 0;
    uint8_t* peer[mf::kPlanMaxWorld] = {};
    bool opened[mf::kPlanMaxWorld] = {};
    bool connected = false;
    int32_t epoch = 0;
    // the two-launch form: the caller's chunk table, the exchange descriptor, and
    // whether a run's amax pass is waiting for its cast pass
    std::vector<mf_chunk_desc> table;
    mf::AmaxXchg* d_xchg = nullptr;
    bool pending = false;
};

using namespace mf;

namespace {

void plan_release(mf_ckpt_plan_s* p) {
    if (!p) return;
    for (int r = 0; r < kPlanMaxWorld; ++r)
        if (p->opened[r]) cudaIpcCloseMemHandle(p->peer[r]);
    cudaFree(p->d_chunks);
    cudaFree(p->d_groups);
    cudaFree(p->d_scratch);
    cudaFree(p->d_xbuf);
    cudaFree(p->d_xchg);
    cudaGetLastError();
    delete p;
}

// The two-launch form's exchange descriptor, once every peer buffer is mapped.
cudaError_t upload_xchg(mf_ckpt_plan_s* p) {
    AmaxXchg h{};
    for (int r = 0; r < p->world; ++r) {
        h.flags[r] = reinterpret_cast<int32_t*>(p->peer[r]);
        h.slots[r] = reinterpret_cast<float*>(p->peer[r] + p->slots_off);
    }
    h.local_amax = reinterpret_cast<float*>(p->d_scratch);
    h.counter = reinterpret_cast<int32_t*>(p->d_scratch + p->counter_off);
    h.arrivals = reinterpret_cast<int32_t*>(p->d_scratch + p->arrivals_off);
    h.abandon = reinterpret_cast<int32_t*>(p->d_scratch + p->abandon_off);
    h.world = p->world;
    h.rank = p->rank;
    h.n_tensors = p->n_tensors;
    h.n_groups = p->n_groups;
    return cudaMemcpy(p->d_xchg, &h, sizeof h, cudaMemcpyHostToDevice);
}

}  // namespace

extern "C" int mf_ckpt_plan_create(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                                   const int64_t* tensor_numel, int64_t group_bytes, int32_t world, int32_t rank,
                                   int fp8_dtype, int compat, mf_ckpt_plan* plan, void* ipc_handle) {
    MF_ENTER();
    if (!plan) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: plan is NULL");
    *plan = nullptr;
    if (n_chunks < 0 || n_tensors <= 0 || (n_chunks > 0 && !chunks))
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: bad chunk table (%d chunks, %d tensors)", n_chunks,
                    n_tensors);
    if (world < 1 || world > kPlanMaxWorld || rank < 0 || rank >= world)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: rank %d of world %d (1..%d ranks)", rank, world,
                    kPlanMaxWorld);
    if (world > 1 && !ipc_handle)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: world > 1 needs ipc_handle (64 bytes)");
    if (world > 1 && !tensor_numel)
        return fail(MF_ERR_INVALID_ARGUMENT,
                    "mf_ckpt_plan_create: world > 1 needs tensor_numel (every rank must cut the same groups)");
    if (!is_fp8(fp8_dtype)) return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_ckpt_plan_create: dtype %d is not FP8", fp8_dtype);
    if (compat != MF_COMPAT_REFERENCE && compat != MF_COMPAT_OCP)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: unknown compat mode %d", compat);
    if (group_bytes < 0) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: negative group_bytes");
    int src_dtype = -1;
    std::vector<int64_t> local(n_tensors, 0);
    for (int32_t i = 0; i < n_chunks; ++i) {
        const mf_chunk_desc& d = chunks[i];
        if (d.tensor < 0 || d.tensor >= n_tensors)
            return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: chunk %d names tensor %d of %d", i, d.tensor,
                        n_tensors);
        if (d.n < 0)
            return fail(MF_ERR_SHAPE_INVALID, "mf_ckpt_plan_create: chunk %d has %lld elements", i, (long long)d.n);
        if (!is_float_store_dtype(d.src_dtype))
            return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_ckpt_plan_create: chunk %d source dtype %d unsupported", i,
                        d.src_dtype);
        if (d.n == 0) continue;
        if (!d.src || !d.dst) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_create: chunk %d has a NULL buffer", i);
        if (src_dtype >= 0 && d.src_dtype != src_dtype)
            return fail(MF_ERR_DTYPE_UNSUPPORTED,
                        "mf_ckpt_plan_create: one source dtype per plan (chunk %d is %d, earlier chunks %d); "
                        "use mf_ckpt_quant_fp8 for mixed tables", i, d.src_dtype, src_dtype);
        src_dtype = d.src_dtype;
        local[d.tensor] += d.n;
    }
    if (tensor_numel)
        for (int32_t t = 0; t < n_tensors; ++t)
            if (tensor_numel[t] < 0)
                return fail(MF_ERR_SHAPE_INVALID, "mf_ckpt_plan_create: tensor %d has %lld elements", t,
                            (long long)tensor_numel[t]);
    if (src_dtype < 0) src_dtype = MF_DT_BF16;
    const int in_bytes = src_dtype == MF_DT_F32 ? 4 : 2;
    const int64_t budget = group_bytes > 0 ? group_bytes : kDefaultGroupBytes;

    // groups: consecutive tensors up to the budget of this rank's source bytes,
    // estimated from the global sizes so that every rank cuts the same groups
    std::vector<PlanGroup> groups;
    std::vector<int32_t> group_of(n_tensors);
    {
        int64_t acc = 0;
        PlanGroup cur{0, 0, 0, 0, 0, 0};
        for (int32_t t = 0; t < n_tensors; ++t) {
            const int64_t numel = tensor_numel ? tensor_numel[t] : local[t] * world;
            const int64_t w = (numel + world - 1) / world * in_bytes;
            if (t > cur.t0 && acc + w > budget) {
                cur.t1 = t;
                groups.push_back(cur);
                cur = PlanGroup{t, t, 0, 0, 0, 0};
                acc = 0;
            }
            acc += w;
            group_of[t] = static_cast<int32_t>(groups.size());
        }
        cur.t1 = n_tensors;
        groups.push_back(cur);
    }
    // chunks sorted by group (table order within a group), tiles numbered per group
    int smem_bytes = 0;
    int64_t tile_elems = 0;
    PlanKernel kernel = pick_kernel(src_dtype, fp8_dtype, compat, &smem_bytes, &tile_elems);
    std::vector<int32_t> order;
    for (int32_t i = 0; i < n_chunks; ++i)
        if (chunks[i].n > 0) order.push_back(i);
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t x, int32_t y) { return group_of[chunks[x].tensor] < group_of[chunks[y].tensor]; });
    std::vector<ChunkRec> recs(order.size());
    int64_t total_tiles = 0, elems = 0;
    for (size_t j = 0, gi = 0; gi < groups.size(); ++gi) {
        PlanGroup& grp = groups[gi];
        grp.c0 = static_cast<int32_t>(j);
        int64_t tiles = 0;
        while (j < order.size() && group_of[chunks[order[j]].tensor] == static_cast<int32_t>(gi)) {
            const mf_chunk_desc& d = chunks[order[j]];
            ChunkRec& r = recs[j];
            r.src = d.src;
            r.dst = d.dst;
            r.n = d.n;
            r.tile_begin = tiles;
            r.tensor = d.tensor;
            r.aligned = (aligned16(d.src) && aligned16(d.dst)) ? 1 : 0;
            tiles += (d.n + tile_elems - 1) / tile_elems;
            elems += d.n;
            ++j;
        }
        grp.c1 = static_cast<int32_t>(j);
        grp.tiles = tiles;
        grp.base = total_tiles;
        total_tiles += tiles;
    }

    mf_ckpt_plan_s* p = new mf_ckpt_plan_s();
    p->device = state().device;
    p->world = world;
    p->rank = rank;
    p->n_tensors = n_tensors;
    p->n_groups = static_cast<int>(groups.size());
    p->src_dtype = src_dtype;
    p->fp8 = fp8_dtype;
    p->compat = compat;
    p->kernel = kernel;
    p->smem_bytes = smem_bytes;
    p->total_tiles = total_tiles;
    p->elems = elems;
    auto bail = [&](cudaError_t e, const char* what) {
        plan_release(p);
        return cuda_fail(e, what);
    };
    cudaError_t e;
    const size_t chunk_bytes = std::max<size_t>(1, recs.size()) * sizeof(ChunkRec);
    if ((e = cudaMalloc(&p->d_chunks, chunk_bytes)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: chunk table");
    if (!recs.empty() &&
        (e = cudaMemcpy(p->d_chunks, recs.data(), recs.size() * sizeof(ChunkRec), cudaMemcpyHostToDevice)) != cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: chunk table upload");
    if ((e = cudaMalloc(&p->d_groups, groups.size() * sizeof(PlanGroup))) != cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: group table");
    if ((e = cudaMemcpy(p->d_groups, groups.data(), groups.size() * sizeof(PlanGroup), cudaMemcpyHostToDevice)) !=
        cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: group table upload");
    p->arrivals_off = align256(sizeof(float) * 2 * n_tensors);
    p->abandon_off = p->arrivals_off + align256(sizeof(int32_t) * 2 * groups.size());
    p->counter_off = p->abandon_off + 64;
    const size_t scratch_bytes = p->abandon_off + 256;
    if ((e = cudaMalloc(&p->d_scratch, scratch_bytes)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: scratch");
    if ((e = cudaMemset(p->d_scratch, 0, scratch_bytes)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: scratch");
    p->slots_off = align256(sizeof(int32_t) * groups.size() * world);
    const size_t xbuf_bytes = p->slots_off + align256(sizeof(float) * 2 * world * static_cast<size_t>(n_tensors));
    if ((e = cudaMalloc(&p->d_xbuf, xbuf_bytes)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: exchange buffer");
    if ((e = cudaMemset(p->d_xbuf, 0, xbuf_bytes)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: exchange buffer");
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: set-up");
    if ((e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem_bytes)) != cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: shared memory opt-in");
    int occ = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reinterpret_cast<const void*>(kernel), kStreamBlock,
                                                           smem_bytes)) != cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: occupancy");
    if (occ < 1) {
        plan_release(p);
        return fail(MF_ERR_NEEDS_PLATFORM_SETUP, "mf_ckpt_plan_create: the kernel does not fit on an SM");
    }
    // kPlanCtas CTAs per SM (every CTA stays resident: the launch is cooperative)
    p->grid = state().sm_count * std::min(occ, kPlanCtas);
    p->peer[rank] = p->d_xbuf;
    p->table.assign(chunks, chunks + n_chunks);
    if ((e = cudaMalloc(&p->d_xchg, sizeof(AmaxXchg))) != cudaSuccess)
        return bail(e, "mf_ckpt_plan_create: exchange descriptor");
    if (world > 1) {
        cudaIpcMemHandle_t h;
        if ((e = cudaIpcGetMemHandle(&h, p->d_xbuf)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: IPC handle");
        std::memcpy(ipc_handle, &h, sizeof h);
    } else {
        if ((e = upload_xchg(p)) != cudaSuccess) return bail(e, "mf_ckpt_plan_create: exchange descriptor upload");
        p->connected = true;
    }
    *plan = p;
    return MF_OK;
}

extern "C" int mf_ckpt_plan_connect(mf_ckpt_plan plan, const void* ipc_handles) {
    MF_ENTER();
    if (!plan) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_connect: plan is NULL");
    if (plan->world == 1 || plan->connected) return MF_OK;
    if (!ipc_handles) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_connect: NULL handle table");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
    for (int r = 0; r < plan->world; ++r) {
        if (r == plan->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(ipc_handles) + 64 * r, sizeof h);
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(e, "mf_ckpt_plan_connect: cudaIpcOpenMemHandle");
        plan->peer[r] = static_cast<uint8_t*>(ptr);
        plan->opened[r] = true;
    }
    const cudaError_t e = upload_xchg(plan);
    if (e != cudaSuccess) return cuda_fail(e, "mf_ckpt_plan_connect: exchange descriptor upload");
    plan->connected = true;
    return MF_OK;
}

extern "C" int mf_ckpt_plan_run(mf_ckpt_plan plan, float* d_amax, float* d_scale_inv, mf_stream stream) {
    MF_ENTER();
    if (!plan) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run: plan is NULL");
    if (!plan->connected)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run: plan of rank %d is not connected to its %d peers",
                    plan->rank, plan->world - 1);
    if (plan->device != state().device)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run: plan belongs to device %d", plan->device);
    if (plan->pending)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run: run %d's cast pass (mf_ckpt_plan_run_passes) is pending",
                    plan->epoch);
    PlanArgs a{};
    a.chunks = plan->d_chunks;
    a.groups = plan->d_groups;
    a.local_amax = reinterpret_cast<float*>(plan->d_scratch);
    a.arrivals = reinterpret_cast<int32_t*>(plan->d_scratch + plan->arrivals_off);
    a.abandon = reinterpret_cast<int32_t*>(plan->d_scratch + plan->abandon_off);
    a.out_amax = d_amax;
    a.out_scale_inv = d_scale_inv;
    a.status = sticky_status_ptr();
    for (int r = 0; r < plan->world; ++r) {
        a.flags[r] = reinterpret_cast<int32_t*>(plan->peer[r]);
        a.slots[r] = reinterpret_cast<float*>(plan->peer[r] + plan->slots_off);
    }
    a.n_groups = plan->n_groups;
    a.n_tensors = plan->n_tensors;
    a.world = plan->world;
    a.rank = plan->rank;
    a.epoch = plan->epoch + 1;
    void* args[] = {&a};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(plan->kernel), dim3(plan->grid),
                                                      dim3(kStreamBlock), args, plan->smem_bytes,
                                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "mf_ckpt_plan_run launch");
    plan->epoch = a.epoch;
    return MF_OK;
}

extern "C" int mf_ckpt_plan_run_passes(mf_ckpt_plan plan, int passes, float* d_amax, float* d_scale_inv,
                                       mf_stream stream) {
    MF_ENTER();
    if (!plan) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run_passes: plan is NULL");
    if (passes < 1 || passes > 3)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run_passes: passes must be 1 (amax), 2 (cast) or 3, got %d",
                    passes);
    if (!plan->connected)
        return fail(MF_ERR_INVALID_ARGUMENT,
                    "mf_ckpt_plan_run_passes: plan of rank %d is not connected to its %d peers", plan->rank,
                    plan->world - 1);
    if (plan->device != state().device)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run_passes: plan belongs to device %d", plan->device);
    if ((passes & 1) && plan->pending)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run_passes: run %d's cast pass has not run", plan->epoch);
    if (passes == 2 && !plan->pending)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_run_passes: no amax pass to cast from (passes=1 first)");
    const int32_t epoch = (passes & 1) ? plan->epoch + 1 : plan->epoch;
    float* lam = reinterpret_cast<float*>(plan->d_scratch) + static_cast<int64_t>(epoch & 1) * plan->n_tensors;
    const int rc = launch_plan_passes(plan->table.data(), static_cast<int32_t>(plan->table.size()), plan->src_dtype,
                                      plan->d_xchg, lam, plan->world, epoch, passes, d_amax, d_scale_inv, plan->fp8,
                                      plan->compat, static_cast<cudaStream_t>(stream));
    if (rc) return rc;
    plan->epoch = epoch;
    plan->pending = passes == 1;
    return MF_OK;
}

extern "C" int mf_ckpt_plan_info(mf_ckpt_plan plan, int32_t* n_groups, int32_t* grid, int64_t* elements) {
    if (!plan) return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_plan_info: plan is NULL");
    if (n_groups) *n_groups = plan->n_groups;
    if (grid) *grid = plan->grid;
    if (elements) *elements = plan->elems;
    return MF_OK;
}

extern "C" int mf_ckpt_plan_destroy(mf_ckpt_plan plan) {
    if (!plan) return MF_OK;
    MF_ENTER();
    cudaError_t e = cudaDeviceSynchronize();
    plan_release(plan);
    if (e != cudaSuccess) return cuda_fail(e, "mf_ckpt_plan_destroy");
    return MF_OK;
}
