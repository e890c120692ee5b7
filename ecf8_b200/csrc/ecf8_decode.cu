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
constexpr int kTabBits = 12;                            // multi-symbol table width
constexpr int kTabSize = 1 << kTabBits;
constexpr int kMaxSymsPerEntry = 5;                     // 5 nibbles fit in bits 31..12
constexpr int kSlotWords = 9;                           // 72 nibbles >= 64 + 4 overshoot
constexpr int kMaxGroupElems = kThreads * 64;           // one symbol per bit at most
constexpr int kObufWords = (kMaxGroupElems + 32) / 8;   // + 15 head pad, round to 16
constexpr int kLutRows = ECF8_MAX_LUTS - 1;             // decode rows (row 0 + prefixes)

struct alignas(16) Smem {
    uint32_t tab[kTabSize];                  // multi-symbol entries
    uint32_t slot[kThreads * kSlotWords];    // per-window decoded nibbles (MSB first)
    uint32_t obuf[kObufWords];               // output-ordered exponent nibbles
    uint16_t tmask[kTabSize];                // start offsets of the symbols of an entry
    uint8_t lut[kLutRows * 256];             // reference LUT rows 0..n_luts-2, zero padded
    uint8_t lens[256];                       // reference LUT last row: code lengths
    uint32_t chg[kLutRows * 8];              // per row: bit b set if entry b != entry b-1
    uint32_t wsum[kThreads / 32];            // block-scan warp totals
};
static_assert(offsetof(Smem, obuf) % 16 == 0, "obuf must allow 8-byte vector reads");

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
    int vec_ok;             // encoded/packed 8-byte and out 16-byte aligned
    int pad_;
};

template <int MAXS>
struct Batch {
    long long total_groups;
    int n_streams;
    int pad_;
    DevStream s[MAXS];
};

// ---------------------------------------------------------------------------
// Per-stream set-up: copy the reference LUTs and derive the multi-symbol table.
// Entry layout (u32): bits 31..12 up to five 4-bit symbols, first symbol in
// the top nibble; bits 11..8 the number of stream bits the symbols use; bits
// 4..0 four times the symbol count (so the entry is directly a funnel-shift
// amount).  An entry with count 0 means the first code is longer than 12 bits.
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
// `lo` (lo is a multiple of 2^pad).  A lookup whose key has only its top
// 8 - pad bits known is decided iff this holds.
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

__device__ void build_tables(Smem& S, const DevStream& d) {
    const int t = threadIdx.x;
    for (int i = t; i < kLutRows * 256; i += kThreads) {
        int row = i >> 8;
        S.lut[i] = (row < d.n_luts - 1) ? __ldg(d.luts + i) : (uint8_t)0;
    }
    for (int i = t; i < 256; i += kThreads) S.lens[i] = __ldg(d.luts + (d.n_luts - 1) * 256 + i);
    __syncthreads();
    // Change bitmaps, one ballot per 32 entries (rows are 256 = 8 x 32 wide).
    for (int i = t; i < kLutRows * 256; i += kThreads) {
        const bool change = (i & 255) && S.lut[i] != S.lut[i - 1];
        const uint32_t m = __ballot_sync(0xffffffffu, change);
        if ((t & 31) == 0) S.chg[i >> 5] = m;
    }
    __syncthreads();
    // Multi-symbol entries.  The pattern's 12 bits are followed by unknown
    // bits; a symbol is taken only if every continuation of the known bits
    // gives the same LUT result (carry-forward entries can otherwise map
    // padding to a code that does not match the bits) and its code fits.
    for (int x = t; x < kTabSize; x += kThreads) {
        const uint32_t v = (uint32_t)x << (32 - kTabBits);
        uint32_t syms = 0, mask = 0, pos = 0, c = 0;
        while (c < (uint32_t)kMaxSymsPerEntry) {
            const uint32_t u = v << pos;
            const uint32_t avail = kTabBits - pos;
            const uint32_t b1 = u >> 24;
            if (!row_constant(S, 0, b1, 8 - min(8u, avail))) break;
            uint32_t sym = S.lut[b1];
            if (sym >= 240) {
                const int row = 256 - (int)sym;
                const uint32_t b2 = (u >> 16) & 255u;
                if (!row_constant(S, row, b2, 8 - (avail > 8 ? avail - 8 : 0))) break;
                sym = S.lut[row * 256 + b2];
            }
            const uint32_t len = code_length(S, sym);
            if (pos + len > (uint32_t)kTabBits) break;
            syms |= (sym & 15u) << (28 - 4 * c);
            mask |= 1u << pos;
            pos += len;
            ++c;
        }
        S.tab[x] = syms | (pos << 8) | (4 * c);
        S.tmask[x] = (uint16_t)mask;
    }
}

// ---------------------------------------------------------------------------
// Window decode.  The 64 window bits plus 16 look-ahead bits are kept in a
// left-aligned 64-bit shift register (hi:lo); p is the window bit offset of
// its top.  Decoded nibbles go through a 64-bit accumulator (ah:al) into the
// thread's shared-memory slot, eight at a time.
// ---------------------------------------------------------------------------
struct Decoder {
    uint32_t hi, lo;       // bit register
    uint32_t ah, al;       // nibble accumulator (newest nibble in the low bits)
    uint32_t n4;           // 4 x symbols appended
    uint32_t m4;           // 4 x symbols not yet spilled
    uint32_t* slot;
    int k;                 // words spilled
    int p;                 // window bit offset of the register's top bit
    uint32_t last_idx;     // table index of the last table step
    int last_p;            // window offset of the last step
    bool last_table;       // whether the last step used the table

    __device__ __forceinline__ void step(const Smem& S) {
        const uint32_t idx = hi >> (32 - kTabBits);
        uint32_t e = S.tab[idx];
        uint32_t b = (e >> 8) & 15u;
        last_idx = idx;
        last_p = p;
        last_table = (e & 31u) != 0;
        if (!last_table) {  // first code longer than the table width
            const uint32_t sym = lut_symbol(S, hi);
            b = code_length(S, sym);
            e = ((sym & 15u) << 28) | 4u;
        }
        // append the entry's symbols: shift amount = e & 31 = 4 x count
        ah = __funnelshift_l(al, ah, e);
        al = __funnelshift_l(e, al, e);
        n4 += e & 31u;
        m4 += e & 31u;
        if (m4 >= 32) {
            m4 -= 32;
            slot[k++] = __funnelshift_r(al, ah, m4);
        }
        hi = __funnelshift_l(lo, hi, b);
        lo <<= b;
        p += (int)b;
    }
};

// Decodes the codes that start in window bits [gap, 64) (decode.cu:65-112) and
// returns how many there are; their nibbles are in `slot`.
__device__ __forceinline__ uint32_t decode_window(const Smem& S, uint32_t* slot, uint32_t whi,
                                                  uint32_t wlo, uint32_t la, int gap) {
    Decoder D;
    D.hi = __funnelshift_l(wlo, whi, gap);
    D.lo = wlo << gap;
    D.ah = D.al = 0;
    D.n4 = D.m4 = 0;
    D.slot = slot;
    D.k = 0;
    D.p = gap;
    D.last_idx = 0;
    D.last_p = 0;
    D.last_table = false;
    while (D.p < 16) D.step(S);
    // The register's low p bits are empty: the 16 look-ahead bits go right
    // below the remaining window bits (decode.cu:100).
    D.lo |= la << (D.p - 16);
    while (D.p < 64) D.step(S);
    if (D.m4) slot[D.k] = D.al << (32 - D.m4);
    uint32_t n = D.n4 >> 2;
    // The last table step may have taken symbols that start at or after bit
    // 64; they belong to the next window.
    const int room = 64 - D.last_p;
    if (D.last_table && room < kTabBits) {
        const uint32_t e = S.tab[D.last_idx];
        const uint32_t keep = __popc((uint32_t)S.tmask[D.last_idx] & ((1u << room) - 1u));
        n -= ((e & 31u) >> 2) - keep;
    }
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

__device__ __forceinline__ uint8_t merge1(const Smem& S, const DevStream& d,
                                          unsigned long long base, unsigned long long i) {
    const uint32_t rel = (uint32_t)(i - base);
    const uint32_t e = (S.obuf[rel >> 3] >> (28 - 4 * (rel & 7))) & 15u;
    const uint32_t pb = __ldg(d.packed + (i >> 1));
    const uint32_t n = (i & 1) ? (pb & 15u) : (pb >> 4);
    return (uint8_t)((e << 3) | ((n & 8u) << 4) | (n & 7u));
}

__device__ void decode_group(Smem& S, const DevStream& d, long long g) {
    const int t = threadIdx.x;
    const unsigned long long N = (unsigned long long)d.n_elements;
    // Group g places elements [output_positions[g], output_positions[g+1])
    // (decode.cu:116,144-145,208); an entry the array lacks counts as N.
    unsigned long long start = (g < d.n_op) ? d.op[g] : N;
    unsigned long long end = (g + 1 < d.n_op) ? d.op[g + 1] : N;
    if (end > N) end = N;
    if (start > end) start = end;
    if (end - start > (unsigned long long)kMaxGroupElems) end = start + kMaxGroupElems;
    const unsigned long long base = start & ~15ull;
    const int n_chunks = (int)((end - base + 15) >> 4);
    for (int i = t; i < 2 * n_chunks; i += kThreads) S.obuf[i] = 0;

    // --- window load (decode.cu:42-62) ---
    const long long wi = g * kThreads + t;
    const long long wb = wi * kWindowBytes;
    uint32_t* slot = S.slot + t * kSlotWords;
    uint32_t count = 0;
    if (wb < d.n_bytes) {
        uint32_t whi, wlo, la;
        if (d.vec_ok && wb + kWindowBytes + 2 <= d.n_bytes) {
            const uint2 raw = __ldg(reinterpret_cast<const uint2*>(d.encoded + wb));
            const uint32_t r16 = __ldg(reinterpret_cast<const unsigned short*>(d.encoded + wb + 8));
            whi = __byte_perm(raw.x, 0, 0x0123);
            wlo = __byte_perm(raw.y, 0, 0x0123);
            la = ((r16 & 0xffu) << 8) | (r16 >> 8);
        } else {
            uint32_t b[10];
#pragma unroll
            for (int i = 0; i < 10; ++i) b[i] = (wb + i < d.n_bytes) ? __ldg(d.encoded + wb + i) : 0u;
            whi = (b[0] << 24) | (b[1] << 16) | (b[2] << 8) | b[3];
            wlo = (b[4] << 24) | (b[5] << 16) | (b[6] << 8) | b[7];
            la = (b[8] << 8) | b[9];
        }
        const uint32_t gb = __ldg(d.gaps + (wi >> 1));
        const int gap = (int)((wi & 1) ? (gb & 15u) : (gb >> 4));
        count = decode_window(S, slot, whi, wlo, la, gap);
    }
    // Windows that lie wholly past n_bytes only follow the last real code, so
    // they place nothing; they count 0.

    // --- block exclusive scan of window counts (decode.cu:114-148) ---
    const int lane = t & 31, warp = t >> 5;
    uint32_t v = count;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) S.wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < kThreads / 32 ? S.wsum[lane] : 0u;
#pragma unroll
        for (int o = 1; o < kThreads / 32; o <<= 1) {
            const uint32_t n = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += n;
        }
        if (lane < kThreads / 32) S.wsum[lane] = s;
    }
    __syncthreads();
    const uint32_t excl = v - count + (warp ? S.wsum[warp - 1] : 0u);

    // --- place this window's nibbles in output order ---
    const unsigned long long s0 = start + excl;
    if (count && s0 < end) {
        const int n = (int)min((unsigned long long)count, end - s0);
        const int dpos = (int)(s0 - base);
        const int w0 = dpos >> 3, w1 = (dpos + n - 1) >> 3;
        const int sh = (dpos & 7) * 4;
        const int eoff = (dpos + n) & 7;
        uint32_t prev = 0;
        for (int j = w0, q = 0; j <= w1; ++j, ++q) {
            const uint32_t cur = q < kSlotWords ? slot[q] : 0u;
            uint32_t val = __funnelshift_r(cur, prev, sh);
            prev = cur;
            if (j == w1 && eoff) val &= 0xffffffffu << (32 - 4 * eoff);
            if (j == w0 || j == w1)
                atomicOr(&S.obuf[j], val);
            else
                S.obuf[j] = val;
        }
    }
    __syncthreads();

    // --- merge with sign+mantissa nibbles, 16 elements per store ---
    for (int c = t; c < n_chunks; c += kThreads) {
        const unsigned long long e0 = base + 16ull * c;
        if (d.vec_ok && e0 >= start && e0 + 16 <= end) {
            const uint2 ew = *reinterpret_cast<const uint2*>(&S.obuf[2 * c]);
            const uint2 pw = __ldg(reinterpret_cast<const uint2*>(d.packed + (e0 >> 1)));
            uint4 o;
            merge8(ew.x, pw.x, o.x, o.y);
            merge8(ew.y, pw.y, o.z, o.w);
            *reinterpret_cast<uint4*>(d.out + e0) = o;
        } else {
            const unsigned long long a = e0 < start ? start : e0;
            const unsigned long long b = e0 + 16 < end ? e0 + 16 : end;
            for (unsigned long long i = a; i < b; ++i) d.out[i] = merge1(S, d, base, i);
        }
    }
    __syncthreads();
}

template <int MAXS>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const __grid_constant__ Batch<MAXS> B) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    const long long total = B.total_groups;
    const long long lo = (long long)blockIdx.x * total / gridDim.x;
    const long long hi = (long long)(blockIdx.x + 1) * total / gridDim.x;
    int si = -1;
    for (long long w = lo; w < hi; ++w) {
        int ns = si < 0 ? 0 : si;
        while (w >= B.s[ns].group_begin + B.s[ns].n_groups) ++ns;
        if (ns != si) {
            si = ns;
            build_tables(S, B.s[si]);
            __syncthreads();
        }
        decode_group(S, B.s[si], w - B.s[si].group_begin);
    }
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
    d->vec_ok = aligned(s.encoded, 8) && aligned(s.packed_other_4bits, 8) && aligned(s.outputs, 16);
    d->group_begin = 0;
    d->pad_ = 0;
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
        default: return "unknown status";
    }
}

int ecf8_last_cuda_error(void) { return ecf8::g_last_cuda_error; }

int ecf8_abi_version(void) { return ECF8_ABI_VERSION; }

}  // extern "C"
