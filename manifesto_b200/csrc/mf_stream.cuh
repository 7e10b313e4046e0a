// mf_stream.cuh -- the bulk-copy streaming engine shared by the conversion
// and FP8 cast kernels.
//
// Every element-wise map in this library reads its source once and writes
// its destination once, so its speed is set by how many source bytes are in
// flight per SM.  Issuing plain loads from every thread ties that to the
// register budget and serialises "load, then compute" inside each thread.
// Here one thread per CTA streams the source through a ring of shared-memory
// stages with the Blackwell bulk-copy engine (cp.async.bulk, 1-D, completion
// counted on an mbarrier), kStages tiles ahead of the consumers; all 256
// threads decode the staged tile from shared memory, compute, and write the
// result with 128-bit streaming stores.  The copy engine keeps up to
// kStages x (2 or 3) CTAs x tile bytes of reads in flight per SM without any
// register cost, and the loads of later tiles overlap the compute of the
// current one.
//
// Work is a table of chunks (ChunkRec: src, dst, n, tensor); chunks are cut
// into tiles of stream_tile_elems<source bytes>() elements and every CTA walks a contiguous range
// of tiles (few chunk changes per CTA).  A chunk whose src or dst is not
// 16-byte aligned is processed with plain loads (the producer arrives on the
// stage barrier without a copy).  Ragged chunk ends (n not a multiple of 16)
// are finished with per-element loads.
//
// Waits on an mbarrier are bounded: after kMbarSpinLimit polls the CTA
// records MF_DEVICE_TIMEOUT in the sticky status word, waits (again bounded)
// for the copies it issued, and returns.
#pragma once

#include "mf_async.cuh"
#include "mf_vec.cuh"

namespace mf {

constexpr int kStreamThreads = 256;
constexpr int kConsumerWarps = kStreamThreads / 32;
// Elements per tile for a source format of InBytes bytes per element: 16384
// for 1- and 2-byte formats (16 or 32 KB of source, 4 or 2 stages), 8192 for
// 4-byte ones (32 KB, 2 stages).  A thread meets 8 or 16 lane steps per tile,
// so the per-tile hand-off (mbarrier wait, chunk bookkeeping, fix-up check) is
// paid half as often as with 8192-element tiles: the BF16 checkpoint cast
// measured 9% faster, the FP8 decodes neither faster nor slower, 4096-element
// tiles 10-20% slower everywhere.
template <int InBytes>
constexpr int64_t stream_tile_elems() {
    return InBytes >= 4 ? 8192 : 16384;
}
constexpr int kStreamSmemBudget = 64 * 1024;    // staging bytes per CTA (room for 3 CTAs per SM)
constexpr int kDeviceTimeout = MF_DEVICE_TIMEOUT;  // sticky status code of a timed-out wait

struct ChunkRec {
    const void* src;
    void* dst;
    int64_t n;
    int64_t tile_begin;  // first tile of this chunk within the launch
    int32_t tensor;
    int32_t aligned;     // src, dst (and src2) 16-byte aligned
    const void* src2;    // second source of a two-source op (same element count), else unused
};

struct AmaxXchg;

template <int MaxChunks>
struct StreamArgs {
    const float* amax;   // per-tensor amax (cast ops)
    int* status;         // sticky status word
    int64_t total_tiles;
    int32_t n_chunks;
    int32_t epoch;       // run number of a plan's cast pass (CastXOp), else 0
    const AmaxXchg* xchg;  // the plan's amax exchange (CastXOp), else NULL
    float* out_amax;       // CastXOp writer launch: global amax [n_tensors] (or NULL)
    float* out_scale_inv;  // CastXOp writer launch: scale_inv [n_tensors] (or NULL)
    int32_t writer;        // CastXOp: this launch writes the outputs and clears the next run's scratch
    float scalar;          // the scalar of AxpyOp (alpha) and ScalarOp
    ChunkRec chunk[MaxChunks];
};

// ------------------------------------------- ordering across CTAs and GPUs

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_relaxed_gpu(const float* p) {
    float v;
    asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int32_t ld_relaxed_gpu(const int32_t* p) {
    int32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// The 256 consumer threads of the CTA (named barrier 1; the producer warp never joins).
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kStreamThreads) : "memory"); }

__device__ __forceinline__ float warp_max_f32(float m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

constexpr int kPlanMaxWorld = 8;                          // ranks of a checkpoint plan
constexpr unsigned long long kFlagWaitNs = 2000000000ull;  // bound of a wait on another rank (2 s)

// Per-tensor amax exchange of a checkpoint plan's two-launch form, in device
// memory (written once when the plan is connected).  Every rank owns one
// exchange buffer, opened by the others with CUDA IPC: flags [world] (row 0 of
// the plan's per-group flags) and slots [2][world][n_tensors].  Pass 1's last
// CTA stores this rank's maxima into slot (epoch & 1, rank) of every rank and
// then releases flag `rank` there with the run's epoch; pass 2 acquires all
// flags of its own buffer and takes the maximum over the slots.
struct AmaxXchg {
    float* slots[kPlanMaxWorld];    // rank r's slots (peer mappings; this rank's own buffer at [rank])
    int32_t* flags[kPlanMaxWorld];  // rank r's flags
    float* local_amax;              // [2][n_tensors] this rank's maxima (pass 1 folds into copy epoch & 1)
    int32_t* counter;               // [2] CTAs of the publishing pass-1 launch that finished
    int32_t* arrivals;              // [2][n_groups] the one-launch form's per-run scratch, cleared like it does
    int32_t* abandon;               // [2]
    int32_t world, rank, n_tensors, n_groups;
};

// ------------------------------------------------------------ lane steps
//
// In one step a lane owns kLane consecutive elements (4 or 8) and lane l of
// a warp owns run r0 + l, so a warp step reads and writes one contiguous span
// and every shared and global access is a full vector.  kLane is 8 when both
// element widths are at most 2 bytes (one 16-byte shared read, at most 16
// bytes stored per lane), else 4: a wider per-lane run would split each
// warp's vector accesses over twice the span (half-filled sectors on the
// store side, two-way bank conflicts on the shared side).
template <int InBytes, int OutBytes>
constexpr int lane_elems() { return (InBytes <= 2 && OutBytes <= 2) ? 8 : 4; }

// Bytes (4, 8, 16 or 32) of source elements at p in shared memory -> w.
template <int Bytes>
__device__ __forceinline__ void load_lane_smem(const uint8_t* p, uint32_t (&w)[Bytes / 4]) {
    if constexpr (Bytes == 4) {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else if constexpr (Bytes == 8) {
        const uint2 x = *reinterpret_cast<const uint2*>(p);
        w[0] = x.x;
        w[1] = x.y;
    } else {
#pragma unroll
        for (int k = 0; k < Bytes / 16; ++k) {
            const uint4 x = reinterpret_cast<const uint4*>(p)[k];
            w[4 * k + 0] = x.x;
            w[4 * k + 1] = x.y;
            w[4 * k + 2] = x.z;
            w[4 * k + 3] = x.w;
        }
    }
}

// Bytes (4, 8, 16 or 32) of encoded elements from w to global memory, streaming stores.
template <int Bytes>
__device__ __forceinline__ void store_lane_stream(void* p, const uint32_t (&w)[Bytes / 4]) {
    if constexpr (Bytes == 4) {
        asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(w[0]) : "memory");
    } else if constexpr (Bytes == 8) {
        asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(w[0]), "r"(w[1]) : "memory");
    } else {
#pragma unroll
        for (int k = 0; k < Bytes / 16; ++k)
            st_stream(static_cast<uint4*>(p) + k, make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]));
    }
}

// Load and decode one lane step: v[k] = elements 4k .. 4k+3 (k < Q = kLane / 4).
template <int SRC, int Q>
__device__ __forceinline__ void load_decode_lane(const uint8_t* sp, float (&v)[2][4]) {
    constexpr int kIn = dtype_bytes(SRC);
    uint32_t w[Q * kIn];
    load_lane_smem<4 * Q * kIn>(sp, w);
#pragma unroll
    for (int k = 0; k < Q; ++k) decode4<SRC>(w + k * kIn, v[k]);
}

// ------------------------------------------------------ deferred fix-ups
//
// The reference's FP8 encoders differ from the hardware conversion on a few
// value classes (E4M3: NaN, the subnormal band, 2^-10 exactly; E5M2: NaN, the
// subnormal band, overflow).  On data with many values near zero (activations)
// a quarter to half of all warp steps hold at least one such value, and
// fixing it inline makes the whole warp run the fix-up.  Instead each warp
// parks the lane steps that need it in a 32-slot shared-memory queue (ballot
// + prefix count; the lane skips its store) and encodes the parked steps
// together, one per lane, at a tile end (see kDrainSlots / kDrainTiles) or
// when the queue is full.  A slot keeps its destination address.
constexpr int kFixSlots = 32;

struct FixQueue {
    float4* v;    // this warp's slots: slot i holds a parked step's values in v[2i] (and v[2i+1] for 8 elements)
    uint8_t** d;  // and where its codes go
    uint32_t n;   // filled slots (warp-uniform)
    uint32_t age; // tile ends passed since the oldest parked step (warp-uniform)
};

// When a tile ends, the warp drains its queue once it holds kDrainSlots steps or
// its oldest step has waited kDrainTiles tiles.  Batching several tiles' fix-ups
// into one drain halves their cost on activations (about half of all warp steps
// park one lane there); the age bound keeps every parked store within a few tiles
// of its neighbours, while their lines are still in L2 (on weights, where steps
// park rarely, draining only when full measured slower).  With 16384-element
// tiles a threshold of 8 slots measured 1-2% faster on activations than 16 or 24
// (4, and an age of 2 tiles, the same as 8); the checkpoint cast is unchanged.
constexpr uint32_t kDrainSlots = 8;
constexpr uint32_t kDrainTiles = 4;

// Warp-collective: encode and store every parked step.
template <class Op>
__device__ __forceinline__ void fix_drain(FixQueue& fq) {
    __syncwarp();
    const uint32_t lane = threadIdx.x & 31;
    if (lane < fq.n) Op::fix(fq.v[2 * lane], fq.v[2 * lane + 1], fq.d[lane]);
    __syncwarp();
    fq.n = 0;
    fq.age = 0;
}

// Warp-collective (all 32 lanes): park this lane's step when `fix` is set.
template <class Op, int Q>
__device__ __forceinline__ void fix_push(FixQueue& fq, bool fix, const float (&v)[2][4], uint8_t* d) {
    const uint32_t bal = __ballot_sync(0xffffffffu, fix);
    if (bal == 0u) return;
    const uint32_t cnt = __popc(bal);
    if (fq.n + cnt > kFixSlots) fix_drain<Op>(fq);
    if (fix) {
        const uint32_t slot = fq.n + __popc(bal & ((1u << (threadIdx.x & 31)) - 1u));
#pragma unroll
        for (int k = 0; k < Q; ++k) fq.v[2 * slot + k] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
        fq.d[slot] = d;
    }
    fq.n += cnt;
}

// Encode and store one lane step of FP8 codes at d (reference rules).  DEFER:
// the fix-up goes through the warp's queue (all 32 lanes must be here); else inline.
template <int FP8, int Q, bool DEFER, class Op>
__device__ __forceinline__ void fp8_lane_store(const float (&v)[2][4], uint8_t* d, FixQueue& fq) {
    uint32_t o[Q];
    uint32_t slow = 0u;
#pragma unroll
    for (int k = 0; k < Q; ++k) slow |= encode4_fp8_fast<FP8>(v[k], o[k]);
    if constexpr (DEFER) {
        if (!slow) store_lane_stream<4 * Q>(d, o);
        fix_push<Op, Q>(fq, slow != 0u, v, d);
    } else {
        if (slow) {
#pragma unroll
            for (int k = 0; k < Q; ++k) o[k] = encode4_fp8_ref<FP8>(v[k]);
        }
        store_lane_stream<4 * Q>(d, o);
    }
}

template <int FP8, int Q>
__device__ __forceinline__ void fp8_lane_fix(const float4& a, const float4& b, uint8_t* d) {
    const float v[2][4] = {{a.x, a.y, a.z, a.w}, {b.x, b.y, b.z, b.w}};
    uint32_t o[Q];
#pragma unroll
    for (int k = 0; k < Q; ++k) o[k] = encode4_fp8_ref<FP8>(v[k]);
    store_lane_stream<4 * Q>(d, o);
}

// ----------------------------------------------------------------- ops
//
// step<DEFER>(sp, ch, e, state, fq): elements e .. e+kLane-1 of the chunk,
// whose source bytes are at sp (shared memory).  kDefers: the op parks FP8
// fix-ups in the warp queue when DEFER is set and encodes them in fix().

// Plain conversion src -> dst (mf_convert).
template <int SRC, int DST, int COMPAT>
struct ConvertOp {
    static constexpr int kIn = dtype_bytes(SRC);
    static constexpr int kOut = dtype_bytes(DST);
    static constexpr int kLane = lane_elems<kIn, kOut>();
    static constexpr int kQ = kLane / 4;
    static constexpr bool kDefers = (DST == MF_DT_F8E4M3 || DST == MF_DT_F8E5M2) && COMPAT == 0;
    static constexpr bool kPrologue = false;
    static constexpr int kIn2 = 0;  // one source
    struct State {};
    template <class A>
    __device__ static State setup(const A&, const ChunkRec&) { return {}; }
    template <bool DEFER>
    __device__ static void step(const uint8_t* sp, const ChunkRec& ch, int64_t e, const State&, FixQueue& fq) {
        float v[2][4];
        load_decode_lane<SRC, kQ>(sp, v);
        uint8_t* d = static_cast<uint8_t*>(ch.dst) + e * kOut;
        if constexpr (kDefers) {
            fp8_lane_store<DST, kQ, DEFER, ConvertOp>(v, d, fq);
        } else {
            uint32_t o[kQ * kOut];
#pragma unroll
            for (int k = 0; k < kQ; ++k) encode4<DST>(v[k], o + k * kOut, COMPAT);
            store_lane_stream<kLane * kOut>(d, o);
        }
    }
    __device__ static void fix(const float4& a, const float4& b, uint8_t* d) {
        if constexpr (kDefers) fp8_lane_fix<DST, kQ>(a, b, d);
    }
    __device__ static void element(const ChunkRec& ch, int64_t i, const State&) {
        store_code<DST>(ch.dst, i, encode_f32<DST>(load_as_f32<SRC>(ch.src, i), COMPAT));
    }
};

__host__ __device__ inline float fp8_max_of(int fp8_dtype) { return fp8_dtype == MF_DT_F8E5M2 ? 57344.0f : 448.0f; }

__device__ __forceinline__ float scale_from_amax(float amax, int fp8_dtype) {
    const bool ok = (amax > 0.0f) && (amax < __int_as_float(0x7f800000));
    return ok ? __fdiv_rn(fp8_max_of(fp8_dtype), amax) : 1.0f;
}
__device__ __forceinline__ float scale_inv_from_amax(float amax, int fp8_dtype) {
    const bool ok = (amax > 0.0f) && (amax < __int_as_float(0x7f800000));
    return ok ? __fdiv_rn(amax, fp8_max_of(fp8_dtype)) : 1.0f;
}

__device__ __forceinline__ void scale4(float (&v)[4], float s) {
    const float2 a = __fmul2_rn(make_float2(v[0], v[1]), make_float2(s, s));
    const float2 b = __fmul2_rn(make_float2(v[2], v[3]), make_float2(s, s));
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
}

// Per-tensor amax-scaled FP8 cast: q = encode(v * (fp8_max / amax[tensor])).
template <int SRC, int FP8, int COMPAT>
struct CastOp {
    static constexpr int kIn = dtype_bytes(SRC);
    static constexpr int kLane = lane_elems<kIn, 1>();
    static constexpr int kQ = kLane / 4;
    static constexpr bool kDefers = COMPAT == 0;
    static constexpr bool kPrologue = false;
    static constexpr int kIn2 = 0;
    struct State {
        float scale;
    };
    template <class A>
    __device__ static State setup(const A& a, const ChunkRec& ch) {
        return {scale_from_amax(a.amax[ch.tensor], FP8)};
    }
    template <bool DEFER>
    __device__ static void step(const uint8_t* sp, const ChunkRec& ch, int64_t e, const State& st, FixQueue& fq) {
        float v[2][4];
        load_decode_lane<SRC, kQ>(sp, v);
#pragma unroll
        for (int k = 0; k < kQ; ++k) scale4(v[k], st.scale);
        uint8_t* d = static_cast<uint8_t*>(ch.dst) + e;
        if constexpr (kDefers) {
            fp8_lane_store<FP8, kQ, DEFER, CastOp>(v, d, fq);
        } else {
            uint32_t o[kQ];
#pragma unroll
            for (int k = 0; k < kQ; ++k) encode4<FP8>(v[k], o + k, COMPAT);
            store_lane_stream<4 * kQ>(d, o);
        }
    }
    __device__ static void fix(const float4& a, const float4& b, uint8_t* d) { fp8_lane_fix<FP8, kQ>(a, b, d); }
    __device__ static void element(const ChunkRec& ch, int64_t i, const State& st) {
        store_code<FP8>(ch.dst, i, encode_f32<FP8>(__fmul_rn(load_as_f32<SRC>(ch.src, i), st.scale), COMPAT));
    }
};

// The cast pass of a checkpoint plan's two-launch form: CastOp whose scales
// come from the plan's amax exchange instead of a finished amax vector.  Its
// prologue (the consumer warps, before the first tile; the producer lane is
// already streaming tiles in) waits, bounded, for every rank's flag of this
// run, then takes each of the CTA's chunks' global amax -- the maximum over the
// ranks' slots, or this rank's own maxima on one GPU -- into shared memory.
// CTA 0 of the writer launch also stores the global amax and scale_inv of
// every tensor and clears the next run's per-rank maxima and counter.  A wait
// that runs out records MF_DEVICE_TIMEOUT and the pass completes with the
// slots as they are (the host sees the status; no CTA waits for ever).
template <int SRC, int FP8, int COMPAT, int MaxChunks>
struct CastXOp : CastOp<SRC, FP8, COMPAT> {
    using Base = CastOp<SRC, FP8, COMPAT>;
    using State = typename Base::State;
    static constexpr bool kPrologue = true;
    __device__ static float* table() {
        __shared__ float t[MaxChunks];  // global amax of chunk k0 + i
        return t;
    }
    __device__ static int& first_chunk() {
        __shared__ int k0;
        return k0;
    }
    // set once the prologue is over: the producer lane streams the first ring of
    // tiles in meanwhile, then waits for it (time-bounded like the flag waits)
    // before its first wait for a stage to come back
    __device__ static volatile int& ready() {
        __shared__ int r;
        return r;
    }
    __device__ static void init() { ready() = 0; }
    __device__ static bool await_prologue() {
        const unsigned long long start = globaltimer_ns();
        while (!ready()) {
            if (globaltimer_ns() - start > 2 * kFlagWaitNs) return false;
            __nanosleep(256);
        }
        return true;
    }
    __device__ static float global_amax(const AmaxXchg& x, int par, int t) {
        if (x.world == 1) return ld_relaxed_gpu(x.local_amax + static_cast<int64_t>(par) * x.n_tensors + t);
        float m = 0.0f;
        for (int r = 0; r < x.world; ++r)
            m = fmaxf(m, ld_relaxed_sys(x.slots[x.rank] + (static_cast<int64_t>(par) * x.world + r) * x.n_tensors + t));
        return m;
    }
    template <class A>
    __device__ static void prologue(const A& a, int64_t t0, int64_t t1) {
        const AmaxXchg& x = *a.xchg;
        const int par = a.epoch & 1;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (x.world > 1 && warp == 0) {
            bool ok = true;
            if (lane < x.world) {
                const int32_t* f = x.flags[x.rank] + lane;
                const unsigned long long start = globaltimer_ns();
                // flags only grow; "at least this epoch"
                while (static_cast<int32_t>(static_cast<uint32_t>(ld_acquire_sys(f)) - static_cast<uint32_t>(a.epoch)) < 0) {
                    if (globaltimer_ns() - start > kFlagWaitNs) {
                        ok = false;
                        break;
                    }
                    __nanosleep(64);
                }
            }
            if (!__all_sync(0xffffffffu, ok) && lane == 0) atomicExch(a.status, kDeviceTimeout);
        }
        consumers_sync();
        if (t0 < t1) {
            // the chunks of tiles [t0, t1): one warp per chunk
            int k0 = 0, k1 = a.n_chunks - 1;
            while (k0 < k1) {
                const int mid = (k0 + k1 + 1) >> 1;
                if (a.chunk[mid].tile_begin <= t0) k0 = mid;
                else k1 = mid - 1;
            }
            k1 = k0;
            while (k1 + 1 < a.n_chunks && a.chunk[k1 + 1].tile_begin < t1) ++k1;
            if (threadIdx.x == 0) first_chunk() = k0;
            for (int k = k0 + warp; k <= k1; k += kConsumerWarps)
                if (lane == 0) table()[k - k0] = global_amax(x, par, a.chunk[k].tensor);
        }
        if (blockIdx.x == 0 && a.writer) {
            float* next = x.local_amax + static_cast<int64_t>(par ^ 1) * x.n_tensors;
            for (int t = threadIdx.x; t < x.n_tensors; t += kStreamThreads) {
                const float g = global_amax(x, par, t);
                if (a.out_amax) a.out_amax[t] = g;
                if (a.out_scale_inv) a.out_scale_inv[t] = scale_inv_from_amax(g, FP8);
                next[t] = 0.0f;
            }
            for (int g = threadIdx.x; g < x.n_groups; g += kStreamThreads)
                x.arrivals[static_cast<int64_t>(par ^ 1) * x.n_groups + g] = 0;
            if (threadIdx.x == 0) {
                x.counter[par ^ 1] = 0;
                x.abandon[par ^ 1] = 0;
            }
        }
        consumers_sync();
        if (threadIdx.x == 0) ready() = 1;
    }
    template <class A>
    __device__ static State setup(const A& a, const ChunkRec& ch) {
        const int k = static_cast<int>(&ch - a.chunk);
        return {scale_from_amax(table()[k - first_chunk()], FP8)};
    }
};

// ------------------------------------------------------------- the engine

// A two-source op (kIn2 > 0) stages both sources' tiles side by side in one
// stage: 8192 elements when both are at most 2 bytes wide (32 KB a stage), else
// 4096 -- two stages in the same 64 KB budget.
template <class Op>
constexpr int64_t op_tile_elems() {
    if constexpr (Op::kIn2 == 0) return stream_tile_elems<Op::kIn>();
    else return (Op::kIn + Op::kIn2 <= 4) ? 8192 : 4096;
}

template <class Op>
struct StreamGeometry {
    static constexpr int64_t kTileElems = op_tile_elems<Op>();
    static constexpr int kSrc2Offset = static_cast<int>(kTileElems) * Op::kIn;  // the second source's tile
    static constexpr int kTileBytes = static_cast<int>(kTileElems) * (Op::kIn + Op::kIn2);
    static constexpr int kStages = (kStreamSmemBudget / kTileBytes) < 8 ? (kStreamSmemBudget / kTileBytes) : 8;
    static constexpr int kFixOffset = kStages * kTileBytes + kStages * 16;  // 16-byte aligned
    static constexpr int kFixBytes = Op::kDefers ? kConsumerWarps * kFixSlots * (32 + 8) : 0;
    static constexpr int kSmemBytes = kFixOffset + kFixBytes;
    static_assert(kStages >= 2, "tile too large for the staging budget");
};

template <int MaxChunks>
__device__ __forceinline__ int stream_find_chunk(const StreamArgs<MaxChunks>& a, int64_t t, int from) {
    int k = from;
    while (k + 1 < a.n_chunks && a.chunk[k + 1].tile_begin <= t) ++k;
    return k;
}

template <int MaxChunks>
__device__ __forceinline__ int stream_first_chunk(const StreamArgs<MaxChunks>& a, int64_t t) {
    int lo = 0, hi = a.n_chunks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.chunk[mid].tile_begin <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Warp-specialised pipeline: warps 0..7 consume, warp 8 (one lane) produces.
//   full[s]  completes when the bulk copy of the tile in stage s has landed
//            (1 arrival with the byte count, then the transaction bytes);
//   empty[s] completes when all 8 consumer warps are done with stage s.
// Consumers never synchronise with each other, only with the copy engine.
constexpr int kStreamBlock = kStreamThreads + 32;

template <class Op, int MaxChunks>
__global__ void __launch_bounds__(kStreamBlock, 3) stream_kernel(const __grid_constant__ StreamArgs<MaxChunks> a) {
    using G = StreamGeometry<Op>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kTileBytes);
    uint64_t* empty = full + G::kStages;

    // this CTA's contiguous tile range [t0, t1)
    const int64_t per = a.total_tiles / gridDim.x, extra = a.total_tiles % gridDim.x;
    const int64_t b = blockIdx.x;
    const int64_t t0 = b * per + (b < extra ? b : extra);
    const int64_t t1 = t0 + per + (b < extra ? 1 : 0);
    if (t0 >= t1) {
        // a CTA without tiles still takes part in the op's prologue (CTA 0 may be its writer)
        if constexpr (Op::kPrologue)
            if (threadIdx.x < kStreamThreads) Op::prologue(a, t0, t1);
        return;
    }
    const int64_t ntiles = t1 - t0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
        if constexpr (Op::kPrologue) Op::init();
    }
    __syncthreads();

    if (threadIdx.x >= kStreamThreads) {
        // ---------------- producer: one lane streams tiles into the ring
        if (threadIdx.x != kStreamThreads) return;
        int kp = stream_first_chunk(a, t0);
        int64_t i = 0;
        bool ok = true;
        for (; i < ntiles; ++i) {
            const int s = static_cast<int>(i % G::kStages);
            if constexpr (Op::kPrologue) {
                if (i == G::kStages && !Op::await_prologue()) {
                    ok = false;
                    break;
                }
            }
            if (i >= G::kStages &&
                !mbar_wait(&empty[s], static_cast<uint32_t>((i / G::kStages - 1) & 1))) {
                ok = false;
                break;
            }
            const int64_t t = t0 + i;
            kp = stream_find_chunk(a, t, kp);
            const ChunkRec& ch = a.chunk[kp];
            const int64_t e0 = (t - ch.tile_begin) * G::kTileElems;
            const int64_t cnt = min(G::kTileElems, ch.n - e0);
            const uint32_t bytes = static_cast<uint32_t>((cnt * Op::kIn) & ~int64_t(15));
            if (ch.aligned && bytes > 0) {
                if constexpr (Op::kIn2 > 0) {
                    const uint32_t bytes2 = static_cast<uint32_t>((cnt * Op::kIn2) & ~int64_t(15));
                    mbar_arrive_expect_tx(&full[s], bytes + bytes2);
                    bulk_g2s(smem + s * G::kTileBytes, static_cast<const uint8_t*>(ch.src) + e0 * Op::kIn, bytes,
                             &full[s]);
                    if (bytes2 > 0)
                        bulk_g2s(smem + s * G::kTileBytes + G::kSrc2Offset,
                                 static_cast<const uint8_t*>(ch.src2) + e0 * Op::kIn2, bytes2, &full[s]);
                } else {
                    mbar_arrive_expect_tx(&full[s], bytes);
                    bulk_g2s(smem + s * G::kTileBytes, static_cast<const uint8_t*>(ch.src) + e0 * Op::kIn, bytes,
                             &full[s]);
                }
            } else {
                mbar_arrive(&full[s]);  // consumers read this tile from global memory
            }
        }
        if (!ok) atomicExch(a.status, kDeviceTimeout);
        // Every copy issued must land before the CTA's shared memory goes away:
        // wait (bounded) for the last kStages issued tiles.
        for (int64_t j = (i > G::kStages ? i - G::kStages : 0); j < i; ++j)
            mbar_wait(&full[j % G::kStages], static_cast<uint32_t>((j / G::kStages) & 1));
        return;
    }

    // -------------------- consumers: decode, compute, store
    const int lane = threadIdx.x & 31;
    FixQueue fq;
    fq.v = reinterpret_cast<float4*>(smem + G::kFixOffset) + (threadIdx.x >> 5) * 2 * kFixSlots;
    fq.d = reinterpret_cast<uint8_t**>(smem + G::kFixOffset + kConsumerWarps * kFixSlots * 32) +
           (threadIdx.x >> 5) * kFixSlots;
    fq.n = 0;
    fq.age = 0;
    if constexpr (Op::kPrologue) Op::prologue(a, t0, t1);
    int k = stream_first_chunk(a, t0);
    typename Op::State st = Op::setup(a, a.chunk[k]);
    for (int64_t i = 0; i < ntiles; ++i) {
        const int64_t t = t0 + i;
        const int s = static_cast<int>(i % G::kStages);
        if (a.chunk[k].tile_begin + ((a.chunk[k].n + G::kTileElems - 1) / G::kTileElems) <= t) {
            k = stream_find_chunk(a, t, k);
            st = Op::setup(a, a.chunk[k]);
        }
        const ChunkRec& ch = a.chunk[k];
        const int64_t tile = t - ch.tile_begin;
        const int64_t e0 = tile * G::kTileElems;
        const int64_t cnt = min(G::kTileElems, ch.n - e0);
        // warp-uniform outcome: the lanes meet again in warp-collective fix-up code
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((i / G::kStages) & 1)))) {
            if (lane == 0) atomicExch(a.status, kDeviceTimeout);
            return;  // the producer's own bounded waits end the CTA
        }
        if (ch.aligned) {
            // lane-consecutive runs: every warp access is one contiguous span
            // only the first ((cnt * kIn) & ~15) bytes were copied (16-byte
            // granularity); the elements past them come from global memory
            const uint8_t* tp = smem + s * G::kTileBytes;
            if (cnt == G::kTileElems) {
                // full tile: a fixed trip count, unrolled
                constexpr int kStepsPerThread = static_cast<int>(G::kTileElems / Op::kLane / kStreamThreads);
#pragma unroll
                for (int j = 0; j < kStepsPerThread; ++j) {
                    const int q = threadIdx.x + j * kStreamThreads;
                    if constexpr (Op::kIn2 > 0)
                        Op::step2(tp + q * Op::kLane * Op::kIn, tp + G::kSrc2Offset + q * Op::kLane * Op::kIn2, ch,
                                  e0 + Op::kLane * q, st);
                    else
                        Op::template step<Op::kDefers>(tp + q * Op::kLane * Op::kIn, ch, e0 + Op::kLane * q, st, fq);
                }
                // fill the holes parked steps left in recent tiles' output
                if constexpr (Op::kDefers)
                    if (fq.n && (fq.n >= kDrainSlots || ++fq.age >= kDrainTiles)) fix_drain<Op>(fq);
            } else {
                int copied = static_cast<int>(((cnt * Op::kIn) & ~int64_t(15)) / Op::kIn);
                if constexpr (Op::kIn2 > 0)
                    copied = min(copied, static_cast<int>(((cnt * Op::kIn2) & ~int64_t(15)) / Op::kIn2));
                const int nsteps = copied / Op::kLane;
                for (int q = threadIdx.x; q < nsteps; q += kStreamThreads) {
                    if constexpr (Op::kIn2 > 0)
                        Op::step2(tp + q * Op::kLane * Op::kIn, tp + G::kSrc2Offset + q * Op::kLane * Op::kIn2, ch,
                                  e0 + Op::kLane * q, st);
                    else
                        Op::template step<false>(tp + q * Op::kLane * Op::kIn, ch, e0 + Op::kLane * q, st, fq);
                }
                const int rem = static_cast<int>(cnt) - nsteps * Op::kLane;
                if (threadIdx.x < rem) Op::element(ch, e0 + nsteps * Op::kLane + threadIdx.x, st);
            }
        } else {
            for (int64_t j = e0 + threadIdx.x; j < e0 + cnt; j += kStreamThreads) Op::element(ch, j, st);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // FP8 fix-ups still parked (every warp leaves the loop after the same tiles)
    if constexpr (Op::kDefers)
        if (fq.n) fix_drain<Op>(fq);
}

// Host side: launch the engine over a filled argument block.
int* sticky_status_ptr();

template <class Op, int MaxChunks>
inline cudaError_t launch_stream(const StreamArgs<MaxChunks>& a, int sm_count, cudaStream_t s) {
    using G = StreamGeometry<Op>;
    // per device: resident CTAs per SM after the dynamic shared memory opt-in (0 = not set up yet)
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int resident = 3;
    if (dev >= 0 && dev < 64) {
        if (!per_sm[dev]) {
            cudaError_t e = cudaFuncSetAttribute(stream_kernel<Op, MaxChunks>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
            if (e != cudaSuccess) return e;
            int occ = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, stream_kernel<Op, MaxChunks>, kStreamBlock,
                                                              G::kSmemBytes);
            if (e != cudaSuccess) return e;
            per_sm[dev] = occ < 1 ? 1 : (occ > 3 ? 3 : occ);
        }
        resident = per_sm[dev];
    }
    // A chunk table (the grouped checkpoint passes) runs two CTAs per SM: on the
    // 16 GB checkpoint that step measured 5% faster than three (fewer concurrent
    // sequential streams over the DRAM rows); a single array keeps what fits, which
    // the fix-up-heavy casts of activations need.
    if (MaxChunks > 1 && resident > 2) resident = 2;
    int64_t blocks = static_cast<int64_t>(sm_count) * resident;
    if (a.total_tiles < blocks) blocks = a.total_tiles;
    if (blocks < 1) {
        if constexpr (!Op::kPrologue) return cudaSuccess;
        blocks = 1;  // the prologue still runs (CTA 0 may be the writer)
    }
    stream_kernel<Op, MaxChunks><<<static_cast<unsigned>(blocks), kStreamBlock, G::kSmemBytes, s>>>(a);
    return cudaGetLastError();
}

// One flat array as a single-chunk argument block, cut into tiles of tile_elems.
inline void single_chunk(StreamArgs<1>& a, const void* src, void* dst, int64_t n, bool aligned, int64_t tile_elems) {
    a.chunk[0].src = src;
    a.chunk[0].dst = dst;
    a.chunk[0].n = n;
    a.chunk[0].tile_begin = 0;
    a.chunk[0].tensor = 0;
    a.chunk[0].aligned = aligned ? 1 : 0;
    a.chunk[0].src2 = nullptr;
    a.n_chunks = 1;
    a.total_tiles = (n + tile_elems - 1) / tile_elems;
    a.status = sticky_status_ptr();
}

}  // namespace mf
