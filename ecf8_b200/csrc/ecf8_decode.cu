// ecf8_decode.cu -- sm_100a ECF8 decode engine (product path) and its C ABI.
//
// Decodes the stream format of zeyuyang8/ecf8 (bitstream layout
// dfloat/utils.py:373-499, LUT layout dfloat/utils.py:270-370) bit-exactly
// like the reference kernel dfloat/run/decode.cu:16-211, with a different
// design:
//
//  * Persistent CTAs.  Each CTA of 512 threads walks a contiguous range of
//    4096-byte groups (one reference thread block's worth of stream), across
//    one or many streams of a batch, so per-stream set-up is paid once per
//    CTA, not once per group.
//  * Multi-symbol table.  From the reference's two-level byte LUTs each CTA
//    derives, in shared memory, a 4096-entry table indexed by the next 12
//    stream bits that yields up to five whole symbols, the bits they use and
//    their start offsets.  A window of 64 bits (about 25 symbols for trained
//    weights) costs ~6 dependent lookups instead of ~25 chains of 2-3.
//  * Single decode pass.  The reference decodes every window twice (count,
//    then write).  Here each thread decodes its window once into a private
//    shared-memory slot of nibbles, a warp-shuffle + block scan places every
//    window, and the slots are funnel-shifted into an output-ordered nibble
//    buffer.
//  * Coalesced merge.  The exponent nibbles and the packed sign+mantissa
//    nibbles are merged 16 elements at a time with byte-permute/logic ops and
//    written with one 16-byte store per thread, instead of one byte per thread.
//
// No inter-CTA communication, no global scratch, no allocation.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>
#include <mutex>

#include "ecf8.h"

namespace ecf8 {
namespace {

constexpr int kThreads = ECF8_THREADS_PER_BLOCK;        // windows per group
constexpr int kWindowBytes = ECF8_BYTES_PER_THREAD;     // bytes per window
constexpr int kGroupBytes = kThreads * kWindowBytes;    // 4096
constexpr int kTabBits = 12;                            // multi-symbol table width
constexpr int kTabSize = 1 << kTabBits;
constexpr int kMaxSymsPerEntry = 5;                     // 5 nibbles fit in bits 31..12
constexpr int kSlotWords = 9;                           // 72 nibbles >= 64 + 4 overshoot
constexpr int kMaxGroupElems = kThreads * 64;           // one symbol per bit at most
constexpr int kObufWords = (kMaxGroupElems + 32) / 8;   // + 15 head pad, round to 16
constexpr int kLutRows = ECF8_MAX_LUTS - 1;             // decode rows (row 0 + prefixes)
constexpr int kEncStage = kGroupBytes + 16;             // group bytes + look-ahead, 16-byte units
constexpr int kGapStage = kThreads / 2;                 // 4 bits per window
constexpr int kPackStage = kMaxGroupElems / 2 + 32;     // packed nibbles of one group (+ alignment)

struct alignas(16) Smem {
    uint32_t tab[kTabSize];                  // multi-symbol entries
    uint32_t slot[kThreads * kSlotWords];    // per-window decoded nibbles (MSB first)
    uint32_t obuf[kObufWords];               // output-ordered exponent nibbles
    uint8_t enc[2][kEncStage];               // staged bitstream, double buffered
    uint8_t gaps[2][kGapStage];              // staged gaps, double buffered
    uint8_t pack[kPackStage];                // staged sign+mantissa nibbles
    uint16_t tmask[kTabSize + 8];            // start offsets of an entry's symbols (+ sentinel)
    uint8_t lut[kLutRows * 256];             // reference LUT rows 0..n_luts-2, zero padded
    uint8_t lens[256];                       // reference LUT last row: code lengths
    uint32_t chg[kLutRows * 8];              // per row: bit b set if entry b != entry b-1
    uint32_t wsum[kThreads / 32];            // block-scan warp totals
};
static_assert(offsetof(Smem, obuf) % 16 == 0, "obuf must allow 8-byte vector reads");
static_assert(offsetof(Smem, enc) % 16 == 0 && kEncStage % 16 == 0, "cp.async targets are 16-byte units");
static_assert(offsetof(Smem, gaps) % 16 == 0 && offsetof(Smem, pack) % 16 == 0, "cp.async alignment");

struct DevStream {
    const uint8_t* luts;
    const uint8_t* encoded;
    const uint8_t* packed;
    const uint64_t* op;
    const uint8_t* gaps;
    uint8_t* out;
    long long n_bytes;
    long long n_elements;
    long long n_op;
    long long group_begin;  // first global work index of this stream
    int n_groups;
    int n_luts;
    int async_ok;           // encoded, packed and gaps 16-byte aligned: cp.async staging
    int out16;              // outputs 16-byte aligned: 16-byte stores
};

template <int MAXS>
struct Batch {
    long long total_groups;
    int n_streams;
    int pad_;
    DevStream s[MAXS];
};

// ---------------------------------------------------------------------------
// Staging: global -> shared copies of 16-byte units, zero-filled past `limit`.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Copies bytes [lo, lo + size) of `src` (valid below `limit`) to dst[0, size);
// size is a multiple of 16.  Asynchronous with cp.async when src + lo is
// 16-byte aligned, else plain byte loads.
__device__ __forceinline__ void stage(uint8_t* dst, const uint8_t* src, long long lo, int size, long long limit,
                                      bool async_ok) {
    for (int i = threadIdx.x * 16; i < size; i += kThreads * 16) {
        const long long a = lo + i;
        long long v = limit - a;
        v = v < 0 ? 0 : (v > 16 ? 16 : v);
        if (async_ok) {
            cp_async16(dst + i, v ? src + a : src, (uint32_t)v);
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) dst[i + k] = k < v ? __ldg(src + a + k) : (uint8_t)0;
        }
    }
}

// ---------------------------------------------------------------------------
// Per-stream set-up: copy the reference LUTs and derive the multi-symbol table.
// Entry layout (u32): bits 31..12 up to five 4-bit symbols, first symbol in
// the top nibble; bits 11..8 the number of stream bits the symbols use; bits
// 4..0 four times the symbol count (so the entry is directly a funnel-shift
// amount).  An all-zero entry means no complete code starts the pattern
// within 12 bits; the decoder then uses the two-level LUT directly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lut_symbol(const Smem& S, uint32_t top) {
    // `top` holds the next >= 16 stream bits left-aligned (dfloat/run/decode.cu:86-88).
    uint32_t d = S.lut[top >> 24];
    if (d >= 240) d = S.lut[(256u - d) * 256u + ((top >> 16) & 255u)];
    return d;
}

__device__ __forceinline__ uint32_t code_length(const Smem& S, uint32_t sym) {
    // decode.cu:91.  A length of 0 can only be met in the bits after the EOF
    // code (the reference would spin there); it advances by one bit.
    uint32_t len = S.lens[sym & 255u];
    return len ? len : 1u;
}

// True when LUT row `row` holds one value over the 2^pad entries starting at
// `lo` (lo is a multiple of 2^pad).
__device__ __forceinline__ bool row_constant(const Smem& S, int row, uint32_t lo, uint32_t pad) {
    if (pad == 0) return true;
    const uint32_t* c = S.chg + row * 8;
    if (pad <= 5) {
        const uint32_t n = (1u << pad) - 1u;  // entries after lo
        return (c[lo >> 5] & (((1u << n) - 1u) << ((lo & 31u) + 1u))) == 0;
    }
    uint32_t acc = c[lo >> 5] & ~1u;
    for (uint32_t w = (lo >> 5) + 1; w < (lo >> 5) + (1u << (pad - 5)); ++w) acc |= c[w];
    return acc == 0;
}

// The code at the top of the 16-bit value v, if it is a real code: one whose
// whole code range maps to it in the LUTs.  Every code of the table is one;
// bit patterns of the EOF code or of unused code space are not (there the
// LUT's carry-forward answer depends on bits past the returned length).
__device__ __forceinline__ bool real_code(const Smem& S, uint32_t v, uint32_t& sym, uint32_t& len) {
    const uint32_t b1 = v >> 8;
    const uint32_t d = S.lut[b1];
    if (d < 240) {
        const uint32_t l = S.lens[d];
        if (l == 0 || l > 8) return false;
        if (!row_constant(S, 0, b1 & ~((1u << (8 - l)) - 1u), 8 - l)) return false;
        sym = d;
        len = l;
        return true;
    }
    const int row = 256 - (int)d;
    const uint32_t b2 = v & 255u;
    const uint32_t d2 = S.lut[row * 256 + b2];
    const uint32_t l = S.lens[d2 & 255u];
    if (l <= 8 || l > 16) return false;
    if (!row_constant(S, row, b2 & ~((1u << (16 - l)) - 1u), 16 - l)) return false;
    sym = d2;
    len = l;
    return true;
}

__device__ void build_tables(Smem& S, const DevStream& d) {
    const int t = threadIdx.x;
    for (int i = t; i < kLutRows * 256; i += kThreads) {
        const int row = i >> 8;
        S.lut[i] = (row < d.n_luts - 1) ? __ldg(d.luts + i) : (uint8_t)0;
    }
    for (int i = t; i < 256; i += kThreads) S.lens[i] = __ldg(d.luts + (d.n_luts - 1) * 256 + i);
    if (t < 8) S.tmask[kTabSize + t] = 1;  // start mask of a single directly decoded code
    __syncthreads();
    // Change bitmaps, one ballot per 32 entries (rows are 256 = 8 x 32 wide).
    for (int i = t; i < kLutRows * 256; i += kThreads) {
        const bool change = (i & 255) && S.lut[i] != S.lut[i - 1];
        const uint32_t m = __ballot_sync(0xffffffffu, change);
        if ((t & 31) == 0) S.chg[i >> 5] = m;
    }
    __syncthreads();
    // Entry 0 (all-zero pattern) greedily.
    if (t == 0) {
        uint32_t syms = 0, mask = 0, pos = 0, c = 0, sym, len;
        while (c < (uint32_t)kMaxSymsPerEntry && real_code(S, 0, sym, len) && pos + len <= (uint32_t)kTabBits) {
            syms |= (sym & 15u) << (28 - 4 * c);
            mask |= 1u << pos;
            pos += len;
            ++c;
        }
        S.tab[0] = syms | (pos << 8) | (4 * c);
        S.tmask[0] = (uint16_t)mask;
    }
    __syncthreads();
    // Entry x from entry y = (x << l) & 0xfff, where l is x's first code length:
    // y's codes that end within the remaining 12 - l bits follow.  y has more
    // trailing zeros than x, so entries are built in order of decreasing
    // trailing-zero count, one round per count.
    for (int tz = kTabBits - 1; tz >= 0; --tz) {
        const int n = 1 << (kTabBits - 1 - tz);
        for (int j = t; j < n; j += kThreads) {
            const uint32_t x = (uint32_t)(2 * j + 1) << tz;
            uint32_t sym, len, ent = 0, msk = 0;
            if (real_code(S, x << 4, sym, len) && len <= (uint32_t)kTabBits) {
                uint32_t kept = 0, endk = 0, rest = 0, mrest = 0;
                if (len < (uint32_t)kTabBits) {
                    const uint32_t y = (x << len) & (kTabSize - 1);
                    const uint32_t ey = S.tab[y], my = S.tmask[y];
                    const uint32_t endmask = (ey & 31u) ? ((my & ~1u) | (1u << ((ey >> 8) & 15u))) : 0u;
                    kept = min(__popc(endmask & ((2u << (kTabBits - len)) - 1u)), kMaxSymsPerEntry - 1);
                    if (kept) {
                        endk = __fns(endmask, 0, (int)kept);
                        rest = (ey >> 4) & (((1u << (4 * kept)) - 1u) << (28 - 4 * kept));
                        mrest = my & ((1u << endk) - 1u);
                    }
                }
                ent = ((sym & 15u) << 28) | rest | ((len + endk) << 8) | (4 * (1 + kept));
                msk = 1u | (mrest << len);
            }
            S.tab[x] = ent;
            S.tmask[x] = (uint16_t)msk;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Window decode.  Stream bits [p, 80) of the window (64 bits + 16 look-ahead)
// sit left-aligned in the 96-bit shift register (h:m:x).  Decoded nibbles go
// through a 64-bit accumulator (ah:al) into the thread's shared-memory slot,
// eight at a time.  Returns the number of codes that start in bits [gap, 64)
// (decode.cu:65-112).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t decode_window(const Smem& S, uint32_t* slot, uint32_t w0, uint32_t w1,
                                                  uint32_t la, uint32_t gap) {
    uint32_t h = __funnelshift_l(w1, w0, gap);
    uint32_t m = __funnelshift_l(la << 16, w1, gap);
    uint32_t x = (la << 16) << gap;
    uint32_t p = gap, ah = 0, al = 0, m4 = 0;
    uint32_t* sp = slot;
    uint32_t idx, e, b;
    do {
        idx = h >> (32 - kTabBits);
        e = S.tab[idx];
        b = (e >> 8) & 15u;
        if (b == 0) {  // no complete code within the table width: two-level LUT
            const uint32_t sym = lut_symbol(S, h);
            b = code_length(S, sym);
            e = ((sym & 15u) << 28) | 4u;
            idx = kTabSize;
        }
        ah = __funnelshift_l(al, ah, e);  // append e's symbols; shift = e & 31 = 4 x count
        al = __funnelshift_l(e, al, e);
        m4 += e & 31u;
        if (m4 >= 32) {
            m4 -= 32;
            *sp++ = __funnelshift_r(al, ah, m4);
        }
        h = __funnelshift_l(m, h, b);
        m = __funnelshift_l(x, m, b);
        x <<= b;
        p += b;
    } while (p < 64);
    if (m4) *sp = al << (32 - m4);
    uint32_t n = (uint32_t)(sp - slot) * 8 + (m4 >> 2);
    // The last step may have taken codes that start at or after bit 64; they
    // belong to the next window.
    const uint32_t room = 64 - (p - b);
    if (room < (uint32_t)kTabBits)
        n -= ((e & 31u) >> 2) - __popc((uint32_t)S.tmask[idx] & ((1u << room) - 1u));
    return n;
}

// Eight merged e4m3 bytes from eight exponent nibbles (MSB first in `ew`) and
// four packed sign+mantissa bytes (decode.cu:174-175: out = e<<3 | s<<7 | m).
__device__ __forceinline__ void merge8(uint32_t ew, uint32_t pw, uint32_t& lo, uint32_t& hi) {
    const uint32_t q = __byte_perm(ew, 0, 0x0123);  // byte j = e[2j]<<4 | e[2j+1], like pw
    const uint32_t ev = (pw & 0x80808080u) | ((q >> 1) & 0x78787878u) | ((pw >> 4) & 0x07070707u);
    const uint32_t od = ((pw << 4) & 0x80808080u) | ((q << 3) & 0x78787878u) | (pw & 0x07070707u);
    lo = __byte_perm(ev, od, 0x5140);
    hi = __byte_perm(ev, od, 0x7362);
}

// Output range of group g: [output_positions[g], output_positions[g+1])
// (decode.cu:116,144-145,208), an entry the array lacks counting as n_elements.
struct GroupRange {
    unsigned long long start, end;
};

__device__ __forceinline__ GroupRange group_range(const DevStream& d, long long g) {
    const unsigned long long N = (unsigned long long)d.n_elements;
    unsigned long long start = (g < d.n_op) ? __ldg(d.op + g) : N;
    unsigned long long end = (g + 1 < d.n_op) ? __ldg(d.op + g + 1) : N;
    if (end > N) end = N;
    if (start > end) start = end;
    if (end - start > (unsigned long long)kMaxGroupElems) end = start + kMaxGroupElems;
    return {start, end};
}

__device__ __forceinline__ void stage_window_bytes(Smem& S, int buf, const DevStream& d, long long g) {
    stage(S.enc[buf], d.encoded, g * kGroupBytes, kEncStage, d.n_bytes, d.async_ok);
    stage(S.gaps[buf], d.gaps, g * kGapStage, kGapStage, g * kGapStage + kGapStage, d.async_ok);
}

__device__ __forceinline__ int find_stream(const DevStream* s, int from, long long w) {
    while (w >= s[from].group_begin + s[from].n_groups) ++from;
    return from;
}

template <int MAXS>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const __grid_constant__ Batch<MAXS> B) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    const int t = threadIdx.x;
    const long long total = B.total_groups;
    const long long lo = (long long)blockIdx.x * total / gridDim.x;
    const long long hi = (long long)(blockIdx.x + 1) * total / gridDim.x;
    if (lo >= hi) return;

    int si = find_stream(B.s, 0, lo);
    stage_window_bytes(S, 0, B.s[si], lo - B.s[si].group_begin);
    cp_async_commit();
    GroupRange r = group_range(B.s[si], lo - B.s[si].group_begin);
    build_tables(S, B.s[si]);

    for (long long w = lo; w < hi; ++w) {
        const int buf = (int)((w - lo) & 1);
        const DevStream& d = B.s[si];
        const long long g = w - d.group_begin;
        const unsigned long long start = r.start, end = r.end;
        const unsigned long long base = start & ~15ull;
        const int n_chunks = (int)((end - base + 15) >> 4);

        // Stage this group's packed nibbles, the next group's window bytes,
        // and fetch the next group's output range.
        const long long p0 = (long long)(base >> 1) & ~15ll;
        const int psize = (int)((((long long)((base >> 1) + 8 * (unsigned long long)n_chunks) - p0) + 15) & ~15ll);
        stage(S.pack, d.packed, p0, psize, d.n_elements >> 1, d.async_ok);
        cp_async_commit();
        int sn = si;
        if (w + 1 < hi) {
            sn = find_stream(B.s, si, w + 1);
            const long long gn = w + 1 - B.s[sn].group_begin;
            stage_window_bytes(S, buf ^ 1, B.s[sn], gn);
            r = group_range(B.s[sn], gn);
        }
        cp_async_commit();

        for (int i = t; i < 2 * n_chunks; i += kThreads) S.obuf[i] = 0;
        cp_async_wait<2>();  // this group's window bytes
        __syncthreads();

        // --- decode this thread's window ---
        uint32_t* slot = S.slot + t * kSlotWords;
        uint32_t count = 0;
        if ((g * kThreads + t) * (long long)kWindowBytes < d.n_bytes) {
            const uint2 raw = *reinterpret_cast<const uint2*>(S.enc[buf] + t * kWindowBytes);
            const uint32_t r16 = *reinterpret_cast<const unsigned short*>(S.enc[buf] + t * kWindowBytes + 8);
            const uint32_t gb = S.gaps[buf][t >> 1];
            count = decode_window(S, slot, __byte_perm(raw.x, 0, 0x0123), __byte_perm(raw.y, 0, 0x0123),
                                  ((r16 & 0xffu) << 8) | (r16 >> 8), (t & 1) ? (gb & 15u) : (gb >> 4));
        }
        // Windows wholly past n_bytes only follow the last real code: they place nothing.

        // --- block exclusive scan of window counts (decode.cu:114-148) ---
        const int lane = t & 31, warp = t >> 5;
        uint32_t v = count;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        if (lane == 31) S.wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            uint32_t s = lane < kThreads / 32 ? S.wsum[lane] : 0u;
#pragma unroll
            for (int o = 1; o < kThreads / 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            if (lane < kThreads / 32) S.wsum[lane] = s;
        }
        __syncthreads();
        const uint32_t excl = v - count + (warp ? S.wsum[warp - 1] : 0u);

        // --- place this window's nibbles in output order ---
        const unsigned long long s0 = start + excl;
        if (count && s0 < end) {
            const uint32_t n = (uint32_t)min((unsigned long long)count, end - s0);
            const uint32_t dpos = (uint32_t)(s0 - base);
            const uint32_t w0 = dpos >> 3, nw = ((dpos + n - 1) >> 3) - w0;  // words after the first
            const uint32_t sh = (dpos & 7) * 4;
            const uint32_t tail = (dpos + n) & 7 ? 0xffffffffu << (32 - 4 * ((dpos + n) & 7)) : 0xffffffffu;
            uint32_t prev = slot[0];
            uint32_t first = __funnelshift_r(prev, 0u, sh);
            if (nw == 0) first &= tail;
            atomicOr(&S.obuf[w0], first);
            for (uint32_t q = 1; q < nw; ++q) {
                const uint32_t cur = slot[q];
                S.obuf[w0 + q] = __funnelshift_r(cur, prev, sh);
                prev = cur;
            }
            if (nw) {
                const uint32_t cur = nw < kSlotWords ? slot[nw] : 0u;
                atomicOr(&S.obuf[w0 + nw], __funnelshift_r(cur, prev, sh) & tail);
            }
        }
        cp_async_wait<1>();  // this group's packed nibbles
        __syncthreads();

        // --- merge with sign+mantissa nibbles, 16 elements per store ---
        const uint8_t* pk = S.pack + ((base >> 1) - p0);
        for (int c = t; c < n_chunks; c += kThreads) {
            const unsigned long long e0 = base + 16ull * c;
            const uint2 ew = *reinterpret_cast<const uint2*>(&S.obuf[2 * c]);
            const uint2 pw = *reinterpret_cast<const uint2*>(pk + 8 * c);
            uint4 o;
            merge8(ew.x, pw.x, o.x, o.y);
            merge8(ew.y, pw.y, o.z, o.w);
            if (d.out16 && e0 >= start && e0 + 16 <= end) {
                *reinterpret_cast<uint4*>(d.out + e0) = o;
            } else {
                const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    if (e0 + k >= start && e0 + k < end) d.out[e0 + k] = (uint8_t)(ow[k >> 2] >> (8 * (k & 3)));
            }
        }
        __syncthreads();

        if (sn != si) {  // next group belongs to another stream
            si = sn;
            build_tables(S, B.s[si]);
        }
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
thread_local int g_last_cuda_error = 0;

struct DeviceInfo {
    int sms = 0;
    int blocks_per_sm = 0;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::once_flag g_device_once[kMaxDevices];
int g_device_status[kMaxDevices];

int cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return ECF8_ERR_CUDA;
}

int device_info(DeviceInfo* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return ECF8_ERR_UNSUPPORTED;
    std::call_once(g_device_once[dev], [dev]() {
        DeviceInfo info;
        cudaError_t err = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
        const int smem = (int)sizeof(Smem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(decode_kernel<ECF8_MAX_BATCH>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess)
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&info.blocks_per_sm, decode_kernel<1>,
                                                                kThreads, smem);
        g_device_status[dev] = (int)err;
        g_devices[dev] = info;
    });
    if (g_device_status[dev] != cudaSuccess) return cuda_fail((cudaError_t)g_device_status[dev]);
    *out = g_devices[dev];
    if (out->blocks_per_sm < 1) out->blocks_per_sm = 1;
    return ECF8_OK;
}

bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// Validates one stream and fills its device descriptor.  Returns a status.
int make_stream(const ecf8_stream& s, DevStream* d) {
    if (s.n_luts < 2 || s.n_luts > ECF8_MAX_LUTS) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_bytes < 0 || s.n_elements < 0 || (s.n_elements & 1)) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_output_positions < 1 || s.n_gap_bytes < 0) return ECF8_ERR_INVALID_ARGUMENT;
    const long long group_bytes = (long long)kThreads * kWindowBytes;
    const long long groups = (s.n_bytes + group_bytes - 1) / group_bytes;
    if (groups > 0x7fffffffLL) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_elements > 0 && s.n_bytes == 0) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_gap_bytes < groups * (kThreads / 2)) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_elements > 0 &&
        (!s.luts || !s.encoded || !s.packed_other_4bits || !s.output_positions || !s.gaps || !s.outputs))
        return ECF8_ERR_INVALID_ARGUMENT;
    if (!aligned(s.output_positions, 8)) return ECF8_ERR_INVALID_ARGUMENT;  // read as u64
    d->luts = s.luts;
    d->encoded = s.encoded;
    d->packed = s.packed_other_4bits;
    d->op = s.output_positions;
    d->gaps = s.gaps;
    d->out = s.outputs;
    d->n_bytes = s.n_bytes;
    d->n_elements = s.n_elements;
    d->n_op = s.n_output_positions;
    d->n_luts = s.n_luts;
    // A stream with no elements has nothing to place.
    d->n_groups = s.n_elements > 0 ? (int)groups : 0;
    d->async_ok = aligned(s.encoded, 16) && aligned(s.packed_other_4bits, 16) && aligned(s.gaps, 16);
    d->out16 = aligned(s.outputs, 16);
    d->group_begin = 0;
    return ECF8_OK;
}

template <int MAXS>
int launch(const ecf8_stream* streams, int n, cudaStream_t stream) {
    Batch<MAXS> B;
    long long total = 0;
    int m = 0;
    for (int i = 0; i < n; ++i) {
        DevStream d;
        int st = make_stream(streams[i], &d);
        if (st != ECF8_OK) return st;
        if (d.n_groups == 0) continue;
        d.group_begin = total;
        total += d.n_groups;
        B.s[m++] = d;
    }
    if (total == 0) return ECF8_OK;
    B.total_groups = total;
    B.n_streams = m;
    B.pad_ = 0;
    DeviceInfo info;
    int st = device_info(&info);
    if (st != ECF8_OK) return st;
    long long grid = (long long)info.sms * info.blocks_per_sm;
    if (grid > total) grid = total;
    decode_kernel<MAXS><<<(unsigned)grid, kThreads, sizeof(Smem), stream>>>(B);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return ECF8_OK;
}

int check_format(int threads_per_block, int bytes_per_thread) {
    if (threads_per_block != ECF8_THREADS_PER_BLOCK || bytes_per_thread != ECF8_BYTES_PER_THREAD)
        return ECF8_ERR_UNSUPPORTED;
    return ECF8_OK;
}

}  // namespace
}  // namespace ecf8

extern "C" {

int ecf8_decode(const uint8_t* luts, const uint8_t* encoded, const uint8_t* packed_other_4bits,
                const uint64_t* output_positions, const uint8_t* gaps, uint8_t* outputs, int n_luts,
                int64_t n_bytes, int64_t n_elements, int64_t n_output_positions, int64_t n_gap_bytes,
                int threads_per_block, int bytes_per_thread, void* cuda_stream) {
    int st = ecf8::check_format(threads_per_block, bytes_per_thread);
    if (st != ECF8_OK) return st;
    ecf8_stream s;
    s.luts = luts;
    s.n_luts = n_luts;
    s.reserved0 = 0;
    s.encoded = encoded;
    s.n_bytes = n_bytes;
    s.packed_other_4bits = packed_other_4bits;
    s.output_positions = output_positions;
    s.n_output_positions = n_output_positions;
    s.gaps = gaps;
    s.n_gap_bytes = n_gap_bytes;
    s.outputs = outputs;
    s.n_elements = n_elements;
    return ecf8::launch<1>(&s, 1, (cudaStream_t)cuda_stream);
}

int ecf8_decode_batch(const ecf8_stream* streams, int n_streams, int threads_per_block,
                      int bytes_per_thread, void* cuda_stream) {
    int st = ecf8::check_format(threads_per_block, bytes_per_thread);
    if (st != ECF8_OK) return st;
    if (n_streams < 0 || (n_streams > 0 && !streams)) return ECF8_ERR_INVALID_ARGUMENT;
    // Validate everything before launching anything.
    for (int i = 0; i < n_streams; ++i) {
        ecf8::DevStream d;
        st = ecf8::make_stream(streams[i], &d);
        if (st != ECF8_OK) return st;
    }
    for (int i = 0; i < n_streams; i += ECF8_MAX_BATCH) {
        const int n = n_streams - i < ECF8_MAX_BATCH ? n_streams - i : ECF8_MAX_BATCH;
        st = ecf8::launch<ECF8_MAX_BATCH>(streams + i, n, (cudaStream_t)cuda_stream);
        if (st != ECF8_OK) return st;
    }
    return ECF8_OK;
}

const char* ecf8_status_string(int status) {
    switch (status) {
        case ECF8_OK: return "ok";
        case ECF8_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ECF8_ERR_UNSUPPORTED: return "unsupported stream format parameters";
        case ECF8_ERR_CUDA: return "CUDA runtime error";
        case ECF8_ERR_TOO_LARGE:
            return "stream longer than the no-allocation packer's built-in scratch (268,435,456 elements)";
        default: return "unknown status";
    }
}

int ecf8_last_cuda_error(void) { return ecf8::g_last_cuda_error; }

int ecf8_abi_version(void) { return ECF8_ABI_VERSION; }

}  // extern "C"
