// Pipelined FP64 inverse row pass (included by ntt.cu inside pcb::ntt; every prime of the launch below 2^50,
// N = 2^16).
//
// The same transform as inv_rows (FP64 path), restructured so that its input loads never idle the FP64 pipe. A launch
// runs persistent CTAs (3 per SM); each walks a contiguous range of tiles, a tile being 16 consecutive 256-word blocks
// (32 KiB) of one row. Tiles move with the TMA engine's bulk copies (cp.async.bulk, one 32 KiB copy per tile) into two
// shared-memory stages, each completing on its own mbarrier: while a CTA transforms tile t from one stage, tile t + 1
// streams into the other. The pass's input is often another buffer (ModUp's inverse transform reads the ciphertext,
// out of place), which the plain kernel read word by word. The butterfly exchange runs in place in the stage under an
// XOR swizzle (word e of a block at (e & ~15) | ((e ^ (e >> 4)) & 15)), so both the strided and the contiguous views
// of a half-warp hit 16 distinct bank pairs without padding.
//
// Measured (ncu, cold cache, per 111-row chunk at N = 2^16): 32.7 us against 44.0 for inv_rows. The same pipeline on
// the other three passes was slower (forward columns 55.4 against 33.8 us, forward rows about 10 % slower, inverse
// columns 48.6 against 36.7): a column tile is 256 separate 128-byte copies, and the per-tile barriers cost more than
// the latency they hide where the plain kernel already reads its input with coalesced loads.
//
// Waits: one thread waits on a stage's barrier (bounded, mbar_wait) and the CTA learns the outcome through shared
// memory at the barrier that follows, so every thread takes the same path. A wait that ran out is counted in
// g_wait_timeouts (pcb_device_timeouts); the CTA then waits once more (bounded) for each of its copies in flight and
// stops.

constexpr int PIPE_TILE = 4096;  // words per tile
constexpr int PIPE_TILE_BYTES = PIPE_TILE * 8;
constexpr size_t PIPE_SMEM = 2 * PIPE_TILE_BYTES + 256 * sizeof(double2) + 64;  // stages, twiddles, barriers
constexpr int PIPE_CTAS_PER_SM = 3;

__device__ unsigned int g_wait_timeouts;

struct PipeSmem {
    uint64_t* stages;  // [2][PIPE_TILE]
    double2* tw;       // [256]
    uint64_t* bar;     // [2]
    int* flag;         // the waiting thread's outcome
    __device__ __forceinline__ uint64_t* stage(int buf) const { return stages + buf * PIPE_TILE; }
};
__device__ __forceinline__ PipeSmem pipe_smem(unsigned char* raw) {
    PipeSmem s;
    s.stages = (uint64_t*)raw;
    s.tw = (double2*)(raw + 2 * PIPE_TILE_BYTES);
    s.bar = (uint64_t*)(raw + 2 * PIPE_TILE_BYTES + 256 * sizeof(double2));
    s.flag = (int*)(s.bar + 2);
    return s;
}

// swizzled slot of word e (0 .. 255) of a 256-word block
__device__ __forceinline__ int swz(int e) { return (e & ~15) | ((e ^ (e >> 4)) & 15); }

// The CTA's tile range [t0, t1) of T tiles
__device__ __forceinline__ void tile_range(int T, int& t0, int& t1) {
    t0 = (int)((long long)blockIdx.x * T / gridDim.x);
    t1 = (int)((long long)(blockIdx.x + 1) * T / gridDim.x);
}

// Tile j (the CTA's j-th) sits in stage j & 1 and completes phase (j >> 1) & 1 of that stage's barrier. Thread 0
// waits for it; every thread returns the outcome. On a wait that ran out (counted) thread 0 waits once more for it
// and, when tile j + 1's copy was issued, for that one too, so the CTA stops with no copy in flight.
__device__ __forceinline__ bool pipe_wait(const PipeSmem& s, int j, bool next_issued) {
    if (threadIdx.x == 0) {
        const int buf = j & 1;
        const bool ok = mbar_wait(&s.bar[buf], (uint32_t)(j >> 1) & 1);
        if (!ok) {
            atomicAdd(&g_wait_timeouts, 1u);
            mbar_wait(&s.bar[buf], (uint32_t)(j >> 1) & 1);
            if (next_issued) mbar_wait(&s.bar[buf ^ 1], (uint32_t)((j + 1) >> 1) & 1);
        }
        *s.flag = ok;
    }
    __syncthreads();
    return *s.flag != 0;
}

// Row-pass tile: 32 KiB contiguous, one copy by thread 0
__device__ __forceinline__ void pipe_load_row(const PipeSmem& s, int buf, const uint64_t* src) {
    if (threadIdx.x == 0) {
        fence_async_smem();
        mbar_expect(&s.bar[buf], PIPE_TILE_BYTES);
        bulk_load(s.stage(buf), src, PIPE_TILE_BYTES, &s.bar[buf]);
    }
}
__device__ __forceinline__ void pipe_init(const PipeSmem& s) {
    if (threadIdx.x == 0) {
        mbar_init(&s.bar[0], 1);
        mbar_init(&s.bar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();
}

// End of a tile: this thread's stage accesses are ordered before the next bulk copy into the stage, and every thread
// is done with the stage and the twiddles before they are reused
__device__ __forceinline__ void pipe_release() {
    fence_async_smem();
    __syncthreads();
}

// ------------------------------------------------------------------------------------------------ inverse, rows
// GS spans 1 .. 128 inside 256-word blocks, then the inverse twist; the source is the row itself or src + soff (one
// source row). Thread (lb, u) holds words 16 u + k (round 1), then u + 16 k, as inv_rows.
template <int LOGN>
__global__ void __launch_bounds__(THREADS, PIPE_CTAS_PER_SM) inv_rows_p(PcbNttArgs a, int row0, int nrows) {
    constexpr int G = (1 << (LOGN - 8)) / 16;
    extern __shared__ __align__(128) unsigned char raw[];
    const PipeSmem s = pipe_smem(raw);
    const int lb = threadIdx.x / 16, u = threadIdx.x % 16;
    int t0, t1;
    tile_range(nrows * G, t0, t1);
    pipe_init(s);
    pdl_wait();
    pdl_release();
    auto src_of = [&](int t) {
        const int i = row0 + t / G;
        const uint64_t* base = a.soff ? (const uint64_t*)a.src + ((size_t)a.soff[i] << LOGN)
                                      : (const uint64_t*)a.base + ((size_t)a.roff[i] << LOGN);
        return base + (size_t)(t % G) * PIPE_TILE;
    };
    if (t0 < t1) pipe_load_row(s, 0, src_of(t0));
    int pid_loaded = -1;
    FpMod md{0.0, 0.0};
    for (int t = t0, j = 0; t < t1; ++t, ++j) {
        const int buf = j & 1;
        const bool next = t + 1 < t1;
        if (next) pipe_load_row(s, buf ^ 1, src_of(t + 1));
        const int i = row0 + t / G;
        const RowInfo ri = row_of<LOGN>(a, i);
        const int b = (t % G) * 16 + lb;
        if (ri.pid != pid_loaded) {
            s.tw[tw_slot(threadIdx.x)] = pack_pairs<LOGN>(a.iw, ri.pid)[Pack<LOGN>::ROW + threadIdx.x];
            md = mod_of<LOGN, true>(a.pr[ri.pid].p, a.iw, ri.pid);
            pid_loaded = ri.pid;
        }
        const double* twist = pack_twist<LOGN>(a.iw, ri.pid) + (size_t)b * 256;
        prefetch_l2(twist + 16 * u);  // this thread's 128-byte line of the block's inverse twist
        if (!pipe_wait(s, j, next)) return;
        uint64_t* blk = s.stage(buf) + lb * 256;
        // the block landed in natural order; this thread needs words 16 u .. 16 u + 15, which read in place would hit
        // one bank pair 16 times: read the conflict-free view u + 16 k, store it swizzled, read 16 u + k swizzled.
        // Two halves of 8 (groups k < 8 are rewritten only after every thread has read them; groups 8 .. 15 after)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint64_t w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) w[k] = blk[u + 16 * (8 * h + k)];
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 8; ++k) blk[swz(u + 16 * (8 * h + k))] = w[k];
        }
        __syncwarp();
        double x[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) x[k] = to_f(blk[swz(16 * u + k)]);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const int h = 1 << l;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                if (k & h) continue;
                gs(x[k], x[k + h], s.tw[(1 << (7 - l)) + ((k >> (l + 1)) << 4) + u], md, (l & 1) == 0);
            }
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 16; ++k) blk[swz(16 * u + k)] = (uint64_t)__double_as_longlong(x[k]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 16; ++k) x[k] = __longlong_as_double((long long)blk[swz(u + 16 * k)]);
#pragma unroll
        for (int l = 4; l < 8; ++l) {
            const int hk = 1 << (l - 4);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                if (k & hk) continue;
                gs(x[k], x[k + hk], s.tw[(1 << (7 - l)) + (k >> (l - 3))], md, (l & 1) == 0);
            }
        }
        uint64_t* out = ri.row + (size_t)b * 256;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const double tw = __ldg(twist + u + 16 * k);  // the inverse twist gamma_b^-k of word u + 16 k
            store_mid<true>(out + u + 16 * k, mul_f(x[k], tw, __dmul_rn(tw, md.pinv), md.p));
        }
        pipe_release();
    }
}

// ------------------------------------------------------------------------------------------------ forward rows, ModDown
// fwd_rows<LOGN, FP64, epilogue 1> (out = (ex - o) s, one source batch) with the epilogue's source tile staged while
// the butterflies run: the CTA's 16 blocks of the row are 4096 consecutive words of `ex` (32 KiB), which thread 0
// requests with one bulk copy right after the launch dependency is met. The plain kernel reads them only after its
// butterflies, so the row pass's FP64 work and the epilogue's HBM traffic ran one after the other (58 against 35 us
// per 111-row chunk). The output words go back to natural order through the thread's padded exchange slots, so the
// staged words (u + 16 k), the output words and the coalesced stores share one conflict-free layout.
// The wait is bounded like the pipelined pass's: a wait that ran out is counted (pcb_device_timeouts), waited once
// more, and the epilogue then reads `ex` from global memory (the same words).
constexpr size_t MD_STAGE_BYTES = 16 * 256 * 8;
constexpr size_t MD_SMEM = MD_STAGE_BYTES + 64;  // stage, mbarrier, the waiting thread's outcome

template <int LOGN>
__global__ void __launch_bounds__(THREADS, NTT_ROWS_BLOCKS_F) fwd_rows_md(PcbNttArgs a, int row0) {
    __shared__ double sm[16 * BLKPAD];
    __shared__ double2 sw[256];
    extern __shared__ __align__(128) unsigned char raw[];
    uint64_t* stage = (uint64_t*)raw;
    uint64_t* bar = (uint64_t*)(raw + MD_STAGE_BYTES);
    int* flag = (int*)(bar + 1);
    const int i = row0 + blockIdx.y;
    const RowInfo ri = row_of<LOGN>(a, i);
    const uint64_t p = a.pr[ri.pid].p;
    const FpMod md = mod_of<LOGN, true>(p, a.fw, ri.pid);
    sw[tw_slot(threadIdx.x)] = pack_pairs<LOGN>(a.fw, ri.pid)[Pack<LOGN>::ROW + threadIdx.x];
    const int lb = threadIdx.x / 16, u = threadIdx.x % 16;
    const int b = blockIdx.x * 16 + lb;  // 256-word block of the row
    uint64_t* blk = ri.row + (size_t)b * 256;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_init_fence();
    }
    __syncthreads();
    pdl_wait();
    pdl_release();
    const size_t erow = (size_t)a.roff[i] << LOGN;  // the row's offset in ex and eout
    if (threadIdx.x == 0) {
        fence_async_smem();
        mbar_expect(bar, MD_STAGE_BYTES);
        bulk_load(stage, (const uint64_t*)a.ex + erow + (size_t)blockIdx.x * 4096, MD_STAGE_BYTES, bar);
    }
    double x[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = load_mid<true>(blk + u + 16 * k);
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const int half = 16 >> (l + 1);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & half) continue;
            ct(x[k], x[k + half], sw[(1 << l) + (k >> (4 - l))], md);
        }
    }
    double* s = sm + lb * BLKPAD;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        round_end(x[k], md);
        s[pad(u + 16 * k)] = x[k];
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = s[pad(16 * u + k)];
#pragma unroll
    for (int l = 4; l < 8; ++l) {
        const int half = 16 >> (l - 3);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & half) continue;
            ct(x[k], x[k + half], sw[(1 << l) + ((k >> (8 - l)) << 4) + u], md);
        }
    }
    // canonical words 16 u + k back through this thread's slots; words u + 16 k read out (the block's 16 threads are
    // one half-warp)
    uint64_t* own = (uint64_t*)s;
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        canon(x[k], md);
        own[pad(16 * u + k)] = bits(x[k]);
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(bar, 0);
        if (!ok) {
            atomicAdd(&g_wait_timeouts, 1u);
            mbar_wait(bar, 0);
        }
        *flag = ok;
    }
    __syncthreads();
    const bool staged = *flag != 0;
    const uint64_t sc = ((const uint64_t*)a.es)[ri.pid], scs = ((const uint64_t*)a.ess)[ri.pid];
    const uint64_t* exg = (const uint64_t*)a.ex + erow + (size_t)b * 256;
    const uint64_t* exs = stage + lb * 256;
    uint64_t* eo = (uint64_t*)a.eout + erow + (size_t)b * 256;
#pragma unroll 4
    for (int k = 0; k < 16; ++k) {
        const int w = u + 16 * k;
        const uint64_t xs = staged ? exs[w] : exg[w];
        eo[w] = epi_word(1, xs, own[pad(w)], 0, sc, scs, p);
    }
}
