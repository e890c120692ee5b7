// ecf8_decode.cu -- sm_100a ECF8 decode engine (product path) and its C ABI.
//
// Decodes the stream format of zeyuyang8/ecf8 (bitstream layout
// dfloat/utils.py:373-499, LUT layout dfloat/utils.py:270-370) bit-exactly
// like the reference kernel dfloat/run/decode.cu:16-211, with a different
// design:
//
//  * Persistent CTAs of independent warps.  One CTA per SM holds one copy of
//    the stream's decode tables in shared memory; each warp decodes its own
//    contiguous run of 4096-byte groups (one reference thread block's worth
//    of stream each), in rounds of 64 windows, so warps never wait for one
//    another inside a stream.  Consecutive groups of a warp are consecutive
//    in the output, so a warp's output buffer flows from group to group and
//    only the first and last chunk of its range are written byte by byte.
//  * Multi-symbol table.  An 8192-entry table indexed by the next 13 stream
//    bits yields up to six whole symbols, the bits they use and their count,
//    plus a counter step that advances the bit position, the output nibble
//    count and the output word index with one add.  It is a pure function of
//    the stream's LUTs: ecf8_build_table() derives it once per stream (at
//    load time) and stores a copy of the LUTs with it; every CTA checks that
//    copy against the stream's LUTs and copies the table into shared memory,
//    or derives the table itself when there is none or it does not match.
//  * Two windows per lane, one decode pass.  Each lane decodes its two
//    adjacent 64-bit windows of the round as one continuous run (the first
//    window's gap gives the start), two table steps per loop iteration,
//    into a private slot of nibbles (slots are interleaved word by word, so
//    the lanes' stores fall in distinct banks); a warp-shuffle scan places
//    each run in the warp's output-ordered nibble buffer.
//  * Loads straight into registers.  A round's bitstream (16 bytes + 4 bytes
//    of look-ahead per lane) and gap byte are loaded into registers while the
//    previous round is placed and merged; the packed sign+mantissa nibbles a
//    round's merge needs are loaded right after its decode, so they are not
//    live (holding registers) during the decode loop, and the round before
//    warms L2 with them (prefetch.global.L2), so those loads wait on L2
//    rather than DRAM.
//  * Merge in whole-warp steps.  Once the nibble buffer holds 512 elements
//    past the merge cursor, each lane merges one 16-element chunk per step
//    (byte-permute/logic ops) and writes it with one 16-byte store; what is
//    left moves to the front of the buffer for the next round.
//  * Launch overlap (opt-in, ECF8_DECODE_OVERLAP_PREVIOUS).  With
//    programmatic dependent launch a decode builds its tables and loads its
//    first round while the stream's previous kernel finishes, and writes
//    outputs only after that kernel has completed (griddepcontrol).
//
// No inter-CTA communication, no global scratch, no allocation, no spin-waits.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>
#include <mutex>

#include "ecf8.h"

#ifndef ECF8_DECODE_WARPS
#define ECF8_DECODE_WARPS 27
#endif

namespace ecf8 {
namespace {

constexpr int kGroupWindows = ECF8_THREADS_PER_BLOCK;   // windows per group (512)
constexpr int kWindowBytes = ECF8_BYTES_PER_THREAD;     // bytes per window (8)
constexpr int kTableThreads = 256;                      // build_table_kernel block size
constexpr int kWarps = ECF8_DECODE_WARPS;               // warps per CTA, each decoding its own groups
constexpr int kThreads = kWarps * 32;                   // CTA size
constexpr int kGroupBytes = kGroupWindows * kWindowBytes;  // 4096
constexpr int kRoundBytes = 64 * kWindowBytes;          // one round: two windows per lane (512 bytes)
constexpr int kRounds = kGroupBytes / kRoundBytes;      // rounds per group (8)
constexpr int kRoundReach = kRoundBytes + 4;            // bytes a round reads (look-ahead word of lane 31)
constexpr int kGapStage = kGroupWindows / 2;            // gap bytes per group
constexpr int kRoundGaps = kGapStage / kRounds;         // gap bytes per round (32)
constexpr int kTabBits = 13;                            // multi-symbol table width
constexpr int kTabSize = 1 << kTabBits;
constexpr int kMaxSymsPerEntry = 6;                     // 6 nibbles fit in bits 31..8
constexpr int kSlotWords = 19;                          // 152 nibbles >= 128 + 12 overshoot
constexpr int kMaxGroupElems = kGroupWindows * 64;      // one symbol per bit at most
constexpr int kLutRows = ECF8_MAX_LUTS - 1;             // decode rows (row 0 + prefixes)
constexpr int kStep = 512;                              // elements per merge step (32 lanes x 16)
// Nibble buffer: up to kStep - 1 pending elements plus one round's codes
// (at most one per stream bit), 8 per word.
constexpr int kObufWords = (kStep + kRoundBytes * 8) / 8;
constexpr int kMaxSmem = 232448;                        // opt-in shared memory per CTA (227 KB)

// Prepared table (ECF8_TABLE_BYTES): entries, end-offset masks, a copy of the
// LUTs it was derived from, and a header.
constexpr int kTabEntryOff = 0;
constexpr int kTabEndsOff = kTabSize * 8;
constexpr int kTabLutOff = kTabEndsOff + kTabSize * 2;
constexpr int kTabHeaderOff = kTabLutOff + ECF8_MAX_LUTS * 256;
constexpr uint32_t kTabMagic = 0x38464345u;  // "ECF8"
static_assert(kTabHeaderOff + 16 == ECF8_TABLE_BYTES, "prepared table layout");

// One warp's buffers.
struct alignas(16) WarpBuf {
    uint32_t slot[kSlotWords * 32];  // per-lane decoded nibbles (MSB first); word w of lane l at [32 w + l]
    uint32_t obuf[kObufWords];       // output-ordered exponent nibbles from the merge cursor on
};
static_assert(offsetof(WarpBuf, obuf) % 16 == 0, "obuf must allow 16-byte accesses");
static_assert(sizeof(WarpBuf) % 16 == 0, "warp buffers stay 16-byte aligned");

struct alignas(16) Smem {
    uint2 tab[kTabSize];                     // multi-symbol entries (x: entry, y: counter step)
    uint16_t ends[kTabSize];                 // per entry: bit j set if a symbol other than the last ends at j
    uint8_t lut[kLutRows * 256];             // reference LUT rows 0..n_luts-2, zero padded
    uint8_t lens[256];                       // reference LUT last row: code lengths
    uint32_t chg[kLutRows * 8];              // per row: bit b set if entry b != entry b-1
    WarpBuf warp[kWarps];
};
static_assert(offsetof(Smem, warp) % 16 == 0 && offsetof(Smem, tab) % 16 == 0 && offsetof(Smem, ends) % 16 == 0,
              "vector copies");
static_assert(sizeof(Smem) <= kMaxSmem, "fits the opt-in shared memory of one CTA");

// Shared-memory layout of build_table_kernel: the decode tables only.
struct alignas(16) TableSmem {
    uint2 tab[kTabSize];
    uint16_t ends[kTabSize];
    uint8_t lut[kLutRows * 256];
    uint8_t lens[256];
    uint32_t chg[kLutRows * 8];
};
static_assert(offsetof(Smem, lut) == offsetof(TableSmem, lut) && offsetof(Smem, chg) == offsetof(TableSmem, chg),
              "the table functions see the same layout");

struct DevStream {
    const uint8_t* luts;
    const uint8_t* encoded;
    const uint8_t* packed;
    const uint64_t* op;
    const uint8_t* gaps;
    uint8_t* out;
    const uint32_t* table;  // prepared table (ECF8_TABLE_BYTES) or null
    long long n_bytes;
    long long n_elements;
    long long n_op;
    long long group_begin;  // first global work index of this stream
    int n_groups;
    int n_luts;
    int enc_vec;            // encoded 16-byte aligned: 16-byte loads
    int packed_vec;         // packed 8-byte aligned: 8-byte loads
    int out_vec;            // outputs 16-byte aligned: 16-byte stores
    int pad_;
};

// Multipliers of the run decode's address arithmetic, passed at run time
// (always 8, 4, 1): the table and slot addresses and the counter adds are then
// issued as multiply-adds, which go to the FMA pipe and leave the integer ALU
// pipe to the funnel shifts that dominate the loop (1.6 % shorter layer
// decodes than the same arithmetic as shifts and adds on the integer ALU).
struct Mul {
    uint32_t entry, word, one, pad_;
};

template <int MAXS>
struct Batch {
    long long total_groups;
    int n_streams;
    int pad_;
    Mul mul;
    DevStream s[MAXS];
};

// ---------------------------------------------------------------------------
// Per-stream set-up.  Entry layout (64 bits): x holds up to six 4-bit
// symbols, first symbol in bits 31..28, and the bits they use in bits 4..0
// (directly a funnel-shift amount); y is the counter step: the bits << 23 |
// four times the symbol count.  A pattern with no complete code within the
// 13 bits gets the no-code step (x = 0); the decoder then uses the two-level
// LUT directly.
// ---------------------------------------------------------------------------
template <class SM>
__device__ __forceinline__ uint32_t lut_symbol(const SM& S, uint32_t top) {
    // `top` holds the next >= 16 stream bits left-aligned (dfloat/run/decode.cu:86-88).
    uint32_t d = S.lut[top >> 24];
    if (d >= 240) d = S.lut[(256u - d) * 256u + ((top >> 16) & 255u)];
    return d;
}

template <class SM>
__device__ __forceinline__ uint32_t code_length(const SM& S, uint32_t sym) {
    // decode.cu:91.  A length of 0 can only be met in the bits after the EOF
    // code (the reference would spin there); it advances by one bit.
    uint32_t len = S.lens[sym & 255u];
    return len ? len : 1u;
}

// Bit j set for the end offset of each symbol of entry e (offsets 1..13).
template <class SM>
__device__ __forceinline__ uint32_t entry_ends(const SM& S, uint2 e) {
    const uint32_t c = (e.y & 31u) >> 2;
    uint32_t pos = 0, mask = 0;
    for (uint32_t i = 0; i < c; ++i) {
        pos += code_length(S, (e.x >> (28 - 4 * i)) & 15u);
        mask |= 1u << pos;
    }
    return mask;
}

// True when LUT row `row` holds one value over the 2^pad entries starting at
// `lo` (lo is a multiple of 2^pad).
template <class SM>
__device__ __forceinline__ bool row_constant(const SM& S, int row, uint32_t lo, uint32_t pad) {
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
template <class SM>
__device__ __forceinline__ bool real_code(const SM& S, uint32_t v, uint32_t& sym, uint32_t& len) {
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

// Copies the stream's LUT rows into shared memory (all threads; no barrier).
template <class SM>
__device__ void load_luts(SM& S, const uint8_t* luts, int n_luts) {
    const int t = threadIdx.x;
    for (int i = t; i < kLutRows * 256; i += (int)blockDim.x) {
        const int row = i >> 8;
        S.lut[i] = (row < n_luts - 1) ? __ldg(luts + i) : (uint8_t)0;
    }
    for (int i = t; i < 256; i += (int)blockDim.x) S.lens[i] = __ldg(luts + (n_luts - 1) * 256 + i);
}

// A table entry (64 bits): x = up to six 4-bit symbols, first in bits 31..28,
// with the bits they use in bits 4..0 (the window's funnel-shift amount);
// y = the counter step (bits << 23) | 4 x count (see decode_run), whose low
// five bits are the accumulator's funnel-shift amount.  No complete code
// within the table width: x = 0 and y = kNoCode, a step that only moves the
// bit position past the end of any run, so the run loop exits to its
// long-code path.
constexpr int kPosShift = 23;                          // counter bit position field: bits 31..23
constexpr uint32_t kNoCode = 128u << kPosShift;
constexpr uint32_t kWordField = 0x3ffffu << 5;         // counter word index field: bits 22..5
__device__ __forceinline__ uint2 make_entry(uint32_t syms, uint32_t bits, uint32_t count) {
    return count ? make_uint2(syms | bits, (bits << kPosShift) | (4 * count)) : make_uint2(0u, kNoCode);
}

// A prepared entry as read from memory, with every field the decode relies
// on forced into range (bits 1..kTabBits, count 1..min(bits, kMaxSymsPerEntry)),
// so a table that ecf8_build_table did not write cannot stall a run or make
// it emit more symbols than it has bits.
__device__ __forceinline__ uint2 sanitize_entry(uint2 e) {
    const uint32_t b = e.y >> kPosShift, c4 = e.y & 31u;
    if (b == 0 || b > (uint32_t)kTabBits || c4 == 0 || (c4 & 3u) || c4 > 4u * kMaxSymsPerEntry || c4 > 4u * b)
        return make_uint2(0u, kNoCode);
    return make_entry(e.x & 0xffffff00u, b, c4 >> 2);
}

// Derives the multi-symbol table from the LUTs in shared memory (all threads;
// the LUTs must be visible to every thread).
template <class SM>
__device__ void derive_table(SM& S) {
    const int t = threadIdx.x;
    // Change bitmaps, one ballot per 32 entries (rows are 256 = 8 x 32 wide).
    for (int i = t; i < kLutRows * 256; i += (int)blockDim.x) {
        const bool change = (i & 255) && S.lut[i] != S.lut[i - 1];
        const uint32_t m = __ballot_sync(0xffffffffu, change);
        if ((t & 31) == 0) S.chg[i >> 5] = m;
    }
    __syncthreads();
    // Entry 0 (all-zero pattern) greedily.
    if (t == 0) {
        uint32_t syms = 0, pos = 0, c = 0, sym, len;
        while (c < (uint32_t)kMaxSymsPerEntry && real_code(S, 0, sym, len) && pos + len <= (uint32_t)kTabBits) {
            syms |= (sym & 15u) << (28 - 4 * c);
            pos += len;
            ++c;
        }
        S.tab[0] = make_entry(syms, pos, c);
    }
    __syncthreads();
    // Entry x from entry y = (x << l) mod 2^kTabBits, where l is x's first
    // code length: y's codes that end within the remaining bits follow.  y has
    // more trailing zeros than x, so entries are built in order of decreasing
    // trailing-zero count, one round per count.
    for (int tz = kTabBits - 1; tz >= 0; --tz) {
        const int n = 1 << (kTabBits - 1 - tz);
        for (int j = t; j < n; j += (int)blockDim.x) {
            const uint32_t x = (uint32_t)(2 * j + 1) << tz;
            uint32_t sym, len;
            uint2 ent = make_entry(0u, 0u, 0u);
            if (real_code(S, x << (16 - kTabBits), sym, len) && len <= (uint32_t)kTabBits) {
                uint32_t kept = 0, endk = 0, rest = 0;
                if (len < (uint32_t)kTabBits) {
                    const uint2 ey = S.tab[(x << len) & (kTabSize - 1)];
                    const uint32_t ends = entry_ends(S, ey);
                    kept = min(__popc(ends & ((2u << (kTabBits - len)) - 1u)), kMaxSymsPerEntry - 1);
                    if (kept) {
                        endk = __fns(ends, 0, (int)kept);
                        rest = (ey.x >> 4) & (((1u << (4 * kept)) - 1u) << (28 - 4 * kept));
                    }
                }
                ent = make_entry(((sym & 15u) << 28) | rest, len + endk, 1 + kept);
            }
            S.tab[x] = ent;
        }
        __syncthreads();
    }
}

// Symbol end offsets of every entry but its last symbol's (the run-end fixup
// of decode_run counts the entry's symbols that start before a bit offset).
template <class SM>
__device__ __forceinline__ uint16_t entry_start_mask(const SM& S, uint2 e) {
    return e.x ? (uint16_t)(entry_ends(S, e) & ((1u << (e.y >> kPosShift)) - 1u)) : (uint16_t)0;
}

template <class SM>
__device__ void build_ends(SM& S) {
    for (int i = threadIdx.x; i < kTabSize; i += (int)blockDim.x) S.ends[i] = entry_start_mask(S, S.tab[i]);
    __syncthreads();
}

// LUTs plus the table (all threads; ends with a barrier).  A prepared table is
// used only if it was derived from these very LUTs (its stored copy and
// header match); otherwise, or without one, the CTA derives the table.
__device__ void setup_stream(Smem& S, const DevStream& d) {
    load_luts(S, d.luts, d.n_luts);
    int bad = 1;
    if (d.table) {
        const uint8_t* tb = reinterpret_cast<const uint8_t*>(d.table);
        const uint4* src = reinterpret_cast<const uint4*>(tb + kTabEntryOff);
        uint4* dst = reinterpret_cast<uint4*>(S.tab);
        for (int i = threadIdx.x; i < kTabSize / 2; i += (int)blockDim.x) {
            const uint4 q = __ldg(src + i);
            const uint2 a = sanitize_entry(make_uint2(q.x, q.y)), b = sanitize_entry(make_uint2(q.z, q.w));
            dst[i] = make_uint4(a.x, a.y, b.x, b.y);
        }
        const uint4* esrc = reinterpret_cast<const uint4*>(tb + kTabEndsOff);
        uint4* ends = reinterpret_cast<uint4*>(S.ends);
        for (int i = threadIdx.x; i < kTabSize / 8; i += (int)blockDim.x) ends[i] = __ldg(esrc + i);
        bad = 0;
        if (threadIdx.x == 0) {
            const uint32_t* hdr = reinterpret_cast<const uint32_t*>(tb + kTabHeaderOff);
            bad = __ldg(hdr) != kTabMagic || __ldg(hdr + 1) != (uint32_t)d.n_luts;
        }
        const uint8_t* copy = tb + kTabLutOff;
        for (int i = threadIdx.x; i < d.n_luts * 256; i += (int)blockDim.x)
            bad |= __ldg(copy + i) != __ldg(d.luts + i);
    }
    if (__syncthreads_or(bad)) {  // also makes the LUTs visible to every thread
        derive_table(S);
        build_ends(S);
    }
}

// ---------------------------------------------------------------------------
// Run decode.  A lane's run is its two adjacent windows: stream bits
// [gap, 128) of the pair, with the 32 bits after the pair as look-ahead.  The
// next 160 - p bits sit left-aligned in the shift register h:m:x:y:z.
// Decoded nibbles go through a 64-bit accumulator (ah:al) into the lane's
// slot.  Returns the number of codes that start in run bits [gap, 128) --
// the two windows' counts of decode.cu:65-112 together.
//
// One counter K carries all of a step's bookkeeping: bits 4..0 are the
// nibble bits of the open slot word, bits 22..5 that word's index in the
// slot (carries out of bit 4 advance it), bits 31..23 the bit position p.  A
// table entry's y word is the counter step, so one add does it.  The slot
// store is unconditional (a partly filled word is rewritten until it is
// full).  The loop takes two table steps per iteration and checks the run's
// end once, so its last iteration may run up to two steps past bit 128 (at
// most 12 nibbles past the 128 codes before it: the slot has room for 152).
// A no-code step moves p by 128 (two of them by 256, within the 9-bit field)
// and so leaves the loop, whose exit takes the code from the two-level LUT
// and re-enters; the loop body has no branch of its own.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void lds64(uint32_t a, uint32_t& lo, uint32_t& hi) {
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(lo), "=r"(hi) : "r"(a));
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
// Shared address of the slot word whose index is K's word field, for the
// lane whose word 0 is at lane_s (word w at lane_s + 128 w).
__device__ __forceinline__ uint32_t slot_addr(uint32_t lane_s, uint32_t K) { return lane_s + ((K & kWordField) << 2); }

// w3, w4: the run's stream bytes 12..19 (bits 96..159), for the end fix-up.
__device__ __forceinline__ uint32_t decode_run(const Smem& S, uint32_t lane_s, uint32_t w0, uint32_t w1,
                                               uint32_t w2, uint32_t w3, uint32_t w4, uint32_t gap, Mul M) {
    const uint32_t tab_s = (uint32_t)__cvta_generic_to_shared(S.tab);
    uint32_t h = __funnelshift_l(w1, w0, gap);
    uint32_t m = __funnelshift_l(w2, w1, gap);
    uint32_t x = __funnelshift_l(w3, w2, gap);
    uint32_t y = __funnelshift_l(w4, w3, gap);
    uint32_t z = w4 << gap;
    uint32_t K = gap << kPosShift;
    uint32_t ah = 0, al = 0, elo1, ehi1, elo2, ehi2;
#pragma unroll 1
    for (;;) {
        // Two table steps per iteration: the second looks up the bits after
        // the first's (h1), the register window then moves by both at once.
#pragma unroll 1
        do {
            lds64((h >> (32 - kTabBits)) * M.entry + tab_s, elo1, ehi1);
            const uint32_t h1 = __funnelshift_l(m, h, elo1);
            lds64((h1 >> (32 - kTabBits)) * M.entry + tab_s, elo2, ehi2);
            const uint32_t sa1 = (K & kWordField) * M.word + lane_s;  // slot_addr(lane_s, K)
            ah = __funnelshift_l(al, ah, ehi1);  // append the entry's symbols; shift = ehi & 31 = 4 x count
            al = __funnelshift_l(elo1, al, ehi1);
            K = ehi1 * M.one + K;
            sts32(sa1, __funnelshift_r(al, ah, K));
            const uint32_t sa2 = (K & kWordField) * M.word + lane_s;
            ah = __funnelshift_l(al, ah, ehi2);
            al = __funnelshift_l(elo2, al, ehi2);
            K = ehi2 * M.one + K;
            sts32(sa2, __funnelshift_r(al, ah, K));
            const uint32_t b = elo1 * M.one + elo2;  // low five bits: both steps' bits (at most 26)
            h = __funnelshift_l(m, h, b);
            m = __funnelshift_l(x, m, b);
            x = __funnelshift_l(y, x, b);
            y = __funnelshift_l(z, y, b);
            z = __funnelshift_l(0u, z, b);
        } while (K < (128u << kPosShift));
        if (__builtin_expect(ehi2 != kNoCode, 1)) break;
        // A no-code step (decode.cu:86-91).  If the first step was one, the
        // second read the same bits and was one too; either left everything
        // but the bit position alone.
        if (ehi1 == kNoCode) {
            K -= 2 * kNoCode;
        } else {
            K -= kNoCode;
            if (K >= (128u << kPosShift)) {  // the first step already reached the run's end
                elo2 = ehi2 = 0u;
                break;
            }
        }
        const uint32_t sym = lut_symbol(S, h);
        const uint32_t len = min(code_length(S, sym), 31u);
        elo1 = ((sym & 15u) << 28) | len;
        ehi1 = (len << kPosShift) | 4u;
        elo2 = ehi2 = 0u;
        const uint32_t sa = slot_addr(lane_s, K);
        ah = __funnelshift_l(al, ah, ehi1);
        al = __funnelshift_l(elo1, al, ehi1);
        K += ehi1;
        sts32(sa, __funnelshift_r(al, ah, K));
        h = __funnelshift_l(m, h, elo1);
        m = __funnelshift_l(x, m, elo1);
        x = __funnelshift_l(y, x, elo1);
        y = __funnelshift_l(z, y, elo1);
        z = __funnelshift_l(0u, z, elo1);
        if (K >= (128u << kPosShift)) break;
    }
    const uint32_t m4 = K & 31u;
    const uint32_t words = (K & kWordField) >> 5;
    if (m4) sts32(slot_addr(lane_s, K), al << (32 - m4));
    uint32_t n = words * 8 + (m4 >> 2);
    // The last iteration may have taken codes that start at or after the
    // run's end; they belong to the next run.  Its second step started at p1,
    // its first at p0.  If p1 >= 128 the second step's codes all go and the
    // first step's entry end offsets tell how many of its codes start before
    // the end; otherwise the second step's do.
    const uint32_t p1 = (K >> kPosShift) - (ehi2 >> kPosShift);
    const uint32_t c1 = (ehi1 & 31u) >> 2, c2 = (ehi2 & 31u) >> 2;
    uint32_t q, c, drop;
    if (p1 >= 128u) {
        q = p1 - (ehi1 >> kPosShift);
        c = c1;
        drop = c2;
    } else {
        q = p1;
        c = c2;
        drop = 0u;
    }
    const uint32_t room = 128u - q;
    if (room < (uint32_t)kTabBits) {
        const uint32_t idx = __funnelshift_l(w4, w3, 32u - room) >> (32 - kTabBits);
        const uint32_t keep = min(1u + __popc(S.ends[idx] & ((1u << room) - 1u)), c);
        drop += c - keep;
    }
    n -= min(drop, n);
    return min(n, 128u - gap);  // codes start at distinct bits of [gap, 128); binds only for a corrupt table
}

// Bitwise select: bits of x where m is 1, bits of y where m is 0 (one LOP3).
__device__ __forceinline__ uint32_t bitsel(uint32_t x, uint32_t y, uint32_t m) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(x), "r"(y), "r"(m));
    return r;
}

// Eight merged e4m3 bytes from eight exponent nibbles (MSB first in `ew`) and
// four packed sign+mantissa bytes (decode.cu:174-175: out = e<<3 | s<<7 | m).
// Each output byte takes bit 7 (sign), bits 6..3 (exponent) and bits 2..0
// (mantissa) from three shifted sources, so two selects build it; the masks
// cover every bit, so no source needs masking first.
__device__ __forceinline__ void merge8(uint32_t ew, uint32_t pw, uint32_t& lo, uint32_t& hi) {
    const uint32_t q = __byte_perm(ew, 0, 0x0123);  // byte j = e[2j]<<4 | e[2j+1], like pw
    const uint32_t ev = bitsel(pw, bitsel(pw >> 4, q >> 1, 0x07070707u), 0x80808080u);  // elements 2j
    const uint32_t od = bitsel(pw << 4, bitsel(pw, q << 3, 0x07070707u), 0x80808080u);  // elements 2j+1
    lo = __byte_perm(ev, od, 0x5140);
    hi = __byte_perm(ev, od, 0x7362);
}

__device__ __forceinline__ uint4 merge16(uint2 ew, uint2 p) {
    uint4 o;
    merge8(ew.x, p.x, o.x, o.y);
    merge8(ew.y, p.y, o.z, o.w);
    return o;
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

__device__ __forceinline__ int find_stream(const DevStream* s, int from, long long w) {
    while (w >= s[from].group_begin + s[from].n_groups) ++from;
    return from;
}

// Eight packed bytes of the stream at byte offset `off` (multiple of 8); bytes
// at or past n_elements / 2 read as 0.
__device__ __forceinline__ uint2 packed8(const DevStream& d, unsigned long long off) {
    const unsigned long long limit = (unsigned long long)d.n_elements >> 1;
    if (d.packed_vec && off + 8 <= limit) return __ldg(reinterpret_cast<const uint2*>(d.packed + off));
    uint32_t b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) b[k] = off + k < limit ? __ldg(d.packed + off + k) : 0u;
    return make_uint2(b[0] | b[1] << 8 | b[2] << 16 | b[3] << 24, b[4] | b[5] << 8 | b[6] << 16 | b[7] << 24);
}

// Merges output chunk c (16 elements from base + 16c) and stores the
// elements inside [lo, hi) (relative to base) byte by byte.
__device__ __forceinline__ void store_bytes(const DevStream& d, unsigned long long base, uint32_t c, uint2 ew,
                                            uint2 p, uint32_t lo, uint32_t hi) {
    const uint4 o = merge16(ew, p);
    const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
    uint8_t* dst = d.out + base;
    const uint32_t e0 = 16u * c;
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (e0 + k >= lo && e0 + k < hi) dst[e0 + k] = (uint8_t)(ow[k >> 2] >> (8 * (k & 3)));
}

// Copies run nibbles [dpos, dpos + n) (output positions relative to the
// nibble buffer's word 0) from the lane's slot (word q at slot[32 q]) into
// the buffer.  The run's first and last words are shared with the
// neighbouring runs (atomicOr into the zeroed buffer); the words in between
// are its own.  Reading slot word nw when it is past the run's last written
// word stays inside the slot and is masked off by `tail`.
__device__ __forceinline__ void place_run(uint32_t* obuf, const uint32_t* slot, uint32_t dpos, uint32_t n) {
    const uint32_t e = dpos + n;
    const uint32_t nw = ((e - 1) >> 3) - (dpos >> 3);  // words after the first
    const uint32_t sh = (dpos & 7) * 4;
    const uint32_t tail = 0xffffffffu << (((8u - (e & 7)) * 4) & 31);
    const uint32_t o0 = dpos >> 3;
    uint32_t prev = slot[0];
    atomicOr(obuf + o0, (prev >> sh) & (nw ? 0xffffffffu : tail));
    uint32_t q = 1;
    for (; q + 1 < nw; q += 2) {
        const uint32_t c0 = slot[32 * q], c1 = slot[32 * (q + 1)];
        obuf[o0 + q] = __funnelshift_r(c0, prev, sh);
        obuf[o0 + q + 1] = __funnelshift_r(c1, c0, sh);
        prev = c1;
    }
    if (q < nw) {
        const uint32_t c0 = slot[32 * q];
        obuf[o0 + q] = __funnelshift_r(c0, prev, sh);
        prev = c0;
    }
    if (nw) atomicOr(obuf + o0 + nw, __funnelshift_r(slot[32 * nw], prev, sh) & tail);
}

// One round's input for one lane: its 16 stream bytes plus 4 bytes of
// look-ahead (as loaded: little-endian words of the big-endian stream) and
// its gap byte (the gap of its first window in the high nibble).
struct RoundIn {
    uint32_t w0, w1, w2, w3, w4, gap;
};

// Loads the round at stream byte `lo` with gap bytes `gp`; stream bytes at or
// past n_bytes read as 0.
__device__ __forceinline__ void load_round(RoundIn& in, const DevStream& d, long long lo, const uint8_t* gp,
                                           int lane) {
    in.gap = __ldg(gp + lane);  // gaps exist for every group (n_gap_bytes >= groups x 256)
    const long long off = lo + 16 * lane;
    if (d.enc_vec && lo + kRoundReach <= d.n_bytes) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(d.encoded + off));
        in.w0 = v.x;
        in.w1 = v.y;
        in.w2 = v.z;
        in.w3 = v.w;
        in.w4 = __ldg(reinterpret_cast<const uint32_t*>(d.encoded + off + 16));
    } else {
        uint32_t w[5];
#pragma unroll
        for (int k = 0; k < 5; ++k) {
            uint32_t v = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const long long o = off + 4 * k + j;
                v |= (o < d.n_bytes ? (uint32_t)__ldg(d.encoded + o) : 0u) << (8 * j);
            }
            w[k] = v;
        }
        in.w0 = w[0];
        in.w1 = w[1];
        in.w2 = w[2];
        in.w3 = w[3];
        in.w4 = w[4];
    }
}

// Packed words of chunks C + lane + 32k (k < 4) of the output at `base`,
// those below `climit` (chunks whose 16 elements lie below n_elements); the
// round's merge steps use them.
__device__ __forceinline__ void prefetch_packed(uint2 (&pw)[4], const DevStream& d, unsigned long long base,
                                                uint32_t C, uint32_t climit, int lane) {
    if (d.packed_vec && C + 128 <= climit) {  // all four chunks exist
        const uint2* src = reinterpret_cast<const uint2*>(d.packed + (base >> 1)) + C + lane;
#pragma unroll
        for (int k = 0; k < 4; ++k) pw[k] = __ldg(src + 32 * k);
    } else if (d.packed_vec) {
        const uint2* src = reinterpret_cast<const uint2*>(d.packed + (base >> 1));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t c = C + lane + 32 * k;
            pw[k] = c < climit ? __ldg(src + c) : make_uint2(0u, 0u);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t c = C + lane + 32 * k;
            pw[k] = c < climit ? packed8(d, (base >> 1) + 8ull * c) : make_uint2(0u, 0u);
        }
    }
}

// Merges `steps` whole steps: lane l merges chunks C + l + 32k (k < steps),
// all complete and below n_elements, and zeroes the buffer words it read.
// Chunk 0 is partial when head > 0 (its first `head` elements belong to the
// range before this one) and is written byte by byte.
__device__ __forceinline__ void merge_steps(uint32_t* obuf, const DevStream& d, unsigned long long base,
                                            uint32_t C, uint32_t steps, uint32_t head, int lane,
                                            const uint2 (&pw)[4]) {
    uint2* ew2 = reinterpret_cast<uint2*>(obuf) + lane;
    uint4* ob = reinterpret_cast<uint4*>(d.out + base) + C + lane;
    const uint32_t c0 = C + lane;
    if (d.out_vec && (C || head == 0) && steps <= 4) {  // the common case: no byte stores
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if ((uint32_t)k < steps) {
                const uint2 ew = ew2[32 * k];
                ew2[32 * k] = make_uint2(0u, 0u);
                ob[32 * k] = merge16(ew, pw[k]);
            }
        }
        return;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if ((uint32_t)k < steps) {
            const uint2 ew = ew2[32 * k];
            ew2[32 * k] = make_uint2(0u, 0u);
            const uint32_t c = c0 + 32 * k;
            if (d.out_vec && (c | (head == 0)))
                ob[32 * k] = merge16(ew, pw[k]);
            else
                store_bytes(d, base, c, ew, pw[k], c ? 0u : head, 16u * c + 16u);
        }
    }
    for (uint32_t k = 4; k < steps; ++k) {  // highly compressed rounds only
        const uint2 ew = ew2[32 * k];
        ew2[32 * k] = make_uint2(0u, 0u);
        const uint32_t c = c0 + 32 * k;
        const uint2 p = packed8(d, (base >> 1) + 8ull * c);
        if (d.out_vec)
            ob[32 * k] = merge16(ew, p);
        else
            store_bytes(d, base, c, ew, p, 0u, 16u * c + 16u);
    }
}

// Writes chunks [C, ceil(lim / 16)) of the output at `base`: the pending
// chunks in the buffer, the last one partial, and any chunk past them that
// the codes did not reach (exponent 0); elements below `head` in chunk 0 and
// from `lim` on are left alone.  Zeroes the buffer words it reads.
__device__ void flush_pending(uint32_t* obuf, const DevStream& d, unsigned long long base, uint32_t C,
                              uint32_t lim, uint32_t head, int lane) {
    uint2* ew2 = reinterpret_cast<uint2*>(obuf);
    const uint32_t end = (lim + 15) >> 4;
    for (uint32_t c = C + lane; c < end; c += 32) {
        const uint32_t j = c - C;
        uint2 ew = make_uint2(0u, 0u);
        if (j < (uint32_t)(kObufWords / 2)) {
            ew = ew2[j];
            ew2[j] = make_uint2(0u, 0u);
        }
        const uint32_t lo = c ? 0u : head;
        const uint2 p = packed8(d, (base >> 1) + 8ull * c);
        if (d.out_vec && lo == 0 && 16u * c + 16u <= lim)
            reinterpret_cast<uint4*>(d.out + base)[c] = merge16(ew, p);
        else
            store_bytes(d, base, c, ew, p, lo, lim);
    }
}

// Full 16-element chunks of the output at `base` below n_elements.
__device__ __forceinline__ uint32_t chunk_limit(const DevStream& d, unsigned long long base) {
    const unsigned long long n = ((unsigned long long)d.n_elements - base) >> 4;
    return n > 0x7fffffffull ? 0x7fffffffu : (uint32_t)n;
}

// One warp decodes groups [ga, gb) of stream d, in rounds of 64 windows:
// lane i decodes windows 2i and 2i + 1 of the round as one run into its
// slot, a warp-shuffle scan places the runs after the output position P, and
// whole merge steps are merged and stored.  P, the merge cursor C (a chunk
// index) and the buffer carry from round to round and from group to group;
// all are relative to `base`, the output position (16-aligned) of the
// range's first chunk.  A group that does not start where the previous one
// ended (a stream the reference compressor did not write) flushes the buffer
// and starts a new range.  Only __syncwarp orders the lanes.  Values needed
// only after the decode (the packed words, the next group's range) are
// loaded after it, so the decode loop has the registers to itself.
__device__ void decode_warp(Smem& S, WarpBuf& W, const DevStream& d, int ga, int gb, int lane, Mul M) {
    uint32_t* obuf = W.obuf;
    const uint32_t lane_s = (uint32_t)__cvta_generic_to_shared(W.slot + lane);
    const bool have = ga < gb;
    RoundIn in{};
    uint2 pw[4];
    unsigned long long base = 0;
    uint32_t P = 0, head = 0, re = 0, climit = 0, C = 0;
    // The first round's input is loaded while the CTA sets up the stream's
    // tables (all warps take part; ends with a barrier).
    if (have) {
        const GroupRange rg = group_range(d, ga);
        load_round(in, d, (long long)ga * kGroupBytes, d.gaps + (long long)ga * kGapStage, lane);
        base = rg.start & ~15ull;
        P = head = (uint32_t)(rg.start - base);
        re = (uint32_t)(rg.end - base);
        climit = chunk_limit(d, base);
    }
    setup_stream(S, d);
    // Under programmatic dependent launch (ECF8_DECODE_OVERLAP_PREVIOUS) the
    // set-up above may run while the stream's previous kernel finishes; the
    // outputs are written only after it has completed.  Without that launch
    // attribute this returns at once.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!have) return;

    int g = ga, r = 0;
    long long lo = (long long)ga * kGroupBytes;
#pragma unroll 1
    for (;;) {
        // --- decode this lane's window pair ---
        uint32_t count = 0;
        if (d.n_bytes - lo > 16 * lane)  // a pair wholly past n_bytes only follows the last real code
            count = decode_run(S, lane_s, __byte_perm(in.w0, 0, 0x0123), __byte_perm(in.w1, 0, 0x0123),
                               __byte_perm(in.w2, 0, 0x0123), __byte_perm(in.w3, 0, 0x0123),
                               __byte_perm(in.w4, 0, 0x0123), in.gap >> 4, M);
        prefetch_packed(pw, d, base, C, climit, lane);
        // --- the next round's input: the group's next round, else the next group's first ---
        const bool next_in_group = r + 1 < kRounds && lo + kRoundBytes < d.n_bytes;
        const int gn = next_in_group ? g : g + 1;
        const int rnext = next_in_group ? r + 1 : 0;
        const bool more = gn < gb;
        const long long lon = (long long)gn * kGroupBytes + (long long)rnext * kRoundBytes;
        if (more) load_round(in, d, lon, d.gaps + (long long)gn * kGapStage + rnext * kRoundGaps, lane);

        // --- exclusive scan of run counts (decode.cu:114-148) ---
        uint32_t v = count;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        const uint32_t total = __shfl_sync(0xffffffffu, v, 31);
        const uint32_t dpos = P + v - count;
        const uint32_t n_place = (count && dpos < re) ? min(count, re - dpos) : 0u;
        const uint32_t Pn = min(P + total, re);
        if (n_place) place_run(obuf, W.slot + lane, dpos - 16u * C, n_place);
        __syncwarp();
        // --- whole merge steps, then the rest moves to the buffer's front ---
        const uint32_t steps = (Pn - 16u * C) / kStep;
        if (steps) {
            merge_steps(obuf, d, base, C, steps, head, lane, pw);
            uint2* ew2 = reinterpret_cast<uint2*>(obuf);
            const uint2 t = ew2[32 * steps + lane];
            ew2[32 * steps + lane] = make_uint2(0u, 0u);
            ew2[lane] = t;
            C += 32 * steps;
        }
        // Warm L2 with the packed words the next round's merge steps start
        // from (chunks C .. C + 127): their register loads, issued after the
        // next decode, then wait on L2 rather than DRAM.  A hint only; it
        // holds no register or shared memory across the decode.
        if (more && d.packed_vec) {
            const uint2* src = reinterpret_cast<const uint2*>(d.packed + (base >> 1)) + C + lane;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (C + lane + 32 * k < climit) asm volatile("prefetch.global.L2 [%0];" ::"l"(src + 32 * k));
        }
        __syncwarp();
        P = Pn;
        if (!more) break;
        if (gn != g) {
            // The next group continues this range if it starts where this
            // group ended (always, for a stream the reference compressor
            // wrote); otherwise the range ends here and a new one begins.
            g = gn;
            const GroupRange rg = group_range(d, g);
            if (rg.start < base || rg.start - base != P || P > (1u << 30)) {
                flush_pending(obuf, d, base, C, re, head, lane);
                __syncwarp();
                base = rg.start & ~15ull;
                P = head = (uint32_t)(rg.start - base);
                C = 0;
                climit = chunk_limit(d, base);
            }
            re = (uint32_t)(rg.end - base);
        }
        r = rnext;
        lo = lon;
    }
    flush_pending(obuf, d, base, C, re, head, lane);
    __syncwarp();
}

template <int MAXS>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ Batch<MAXS> B) {
    // A decode launched next with ECF8_DECODE_OVERLAP_PREVIOUS may start its
    // set-up on the SMs this grid leaves; it writes nothing before this grid
    // has completed.
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long total = B.total_groups;
    const long long lo = (long long)blockIdx.x * total / gridDim.x;
    const long long hi = (long long)(blockIdx.x + 1) * total / gridDim.x;
    if (lo >= hi) return;
    // Every warp's nibble buffer starts zeroed and each segment leaves it so.
    WarpBuf& W = S.warp[warp];
    for (int i = lane; i < kObufWords / 4; i += 32) reinterpret_cast<uint4*>(W.obuf)[i] = make_uint4(0, 0, 0, 0);
    __syncwarp();

    // The CTA's range [lo, hi) in per-stream segments: the tables of one
    // stream at a time, each warp taking a contiguous share of the segment.
    int si = find_stream(B.s, 0, lo);
    long long w = lo;
    for (;;) {
        const DevStream& d = B.s[si];
        const long long seg_end = min(hi, d.group_begin + d.n_groups);
        const long long s0 = w - d.group_begin, len = seg_end - w;
        const int ga = (int)(s0 + len * warp / kWarps), gb = (int)(s0 + len * (warp + 1) / kWarps);
        decode_warp(S, W, d, ga, gb, lane, B.mul);
        if (seg_end >= hi) break;
        w = seg_end;
        si = find_stream(B.s, si, w);
        __syncthreads();  // every warp is done with this stream's tables
    }
}

// One CTA derives a stream's multi-symbol table and writes it, with a copy of
// the LUTs and the header, to `table`.
__global__ void __launch_bounds__(kTableThreads, 1) build_table_kernel(const uint8_t* luts, int n_luts,
                                                                       uint32_t* table) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TableSmem& S = *reinterpret_cast<TableSmem*>(smem_raw);
    load_luts(S, luts, n_luts);
    __syncthreads();
    derive_table(S);
    uint8_t* tb = reinterpret_cast<uint8_t*>(table);
    uint2* out = reinterpret_cast<uint2*>(tb + kTabEntryOff);
    uint16_t* ends = reinterpret_cast<uint16_t*>(tb + kTabEndsOff);
    for (int i = threadIdx.x; i < kTabSize; i += (int)blockDim.x) {
        out[i] = S.tab[i];
        ends[i] = entry_start_mask(S, S.tab[i]);
    }
    uint8_t* copy = tb + kTabLutOff;
    for (int i = threadIdx.x; i < ECF8_MAX_LUTS * 256; i += (int)blockDim.x)
        copy[i] = i < n_luts * 256 ? __ldg(luts + i) : (uint8_t)0;
    if (threadIdx.x == 0) {
        uint32_t* hdr = reinterpret_cast<uint32_t*>(tb + kTabHeaderOff);
        hdr[0] = kTabMagic;
        hdr[1] = (uint32_t)n_luts;
        hdr[2] = ECF8_ABI_VERSION;
        hdr[3] = 0;
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
bool g_device_ready[kMaxDevices];
std::mutex g_device_mutex;

int cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return ECF8_ERR_CUDA;
}

// Launch attributes of the current device, set up on its first use.  A failed
// set-up is not remembered: the next call tries again.
int device_info(DeviceInfo* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return ECF8_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (!g_device_ready[dev]) {
        DeviceInfo info;
        const int smem = (int)sizeof(Smem);
        cudaError_t err = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(decode_kernel<ECF8_MAX_BATCH>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(build_table_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(TableSmem));
        if (err == cudaSuccess)
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&info.blocks_per_sm, decode_kernel<1>,
                                                                kThreads, smem);
        if (err != cudaSuccess) return cuda_fail(err);
        if (info.blocks_per_sm < 1) info.blocks_per_sm = 1;
        g_devices[dev] = info;
        g_device_ready[dev] = true;
    }
    *out = g_devices[dev];
    return ECF8_OK;
}

bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// Validates one stream and fills its device descriptor.  Returns a status.
int make_stream(const ecf8_stream& s, DevStream* d) {
    if (s.n_luts < 2 || s.n_luts > ECF8_MAX_LUTS) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_bytes < 0 || s.n_elements < 0 || (s.n_elements & 1)) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_output_positions < 1 || s.n_gap_bytes < 0) return ECF8_ERR_INVALID_ARGUMENT;
    const long long group_bytes = (long long)kGroupBytes;
    const long long groups = (s.n_bytes + group_bytes - 1) / group_bytes;
    if (groups > 0x7fffffffLL) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_elements > 0 && s.n_bytes == 0) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_gap_bytes < groups * kGapStage) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.table && !aligned(s.table, 16)) return ECF8_ERR_INVALID_ARGUMENT;
    if (s.n_elements > 0 &&
        (!s.luts || !s.encoded || !s.packed_other_4bits || !s.output_positions || !s.gaps || !s.outputs))
        return ECF8_ERR_INVALID_ARGUMENT;
    if (!aligned(s.output_positions, 8)) return ECF8_ERR_INVALID_ARGUMENT;  // read as u64
    d->luts = s.luts;
    d->encoded = s.encoded;
    d->packed = s.packed_other_4bits;
    d->op = s.output_positions;
    d->gaps = s.gaps;
    d->table = s.table;
    d->out = s.outputs;
    d->n_bytes = s.n_bytes;
    d->n_elements = s.n_elements;
    d->n_op = s.n_output_positions;
    d->n_luts = s.n_luts;
    // A stream with no elements has nothing to place.
    d->n_groups = s.n_elements > 0 ? (int)groups : 0;
    d->enc_vec = aligned(s.encoded, 16);
    d->packed_vec = aligned(s.packed_other_4bits, 8);
    d->out_vec = aligned(s.outputs, 16);
    d->pad_ = 0;
    d->group_begin = 0;
    return ECF8_OK;
}

int check_format(int threads_per_block, int bytes_per_thread) {
    if (threads_per_block != ECF8_THREADS_PER_BLOCK || bytes_per_thread != ECF8_BYTES_PER_THREAD)
        return ECF8_ERR_UNSUPPORTED;
    return ECF8_OK;
}

// max_ctas: at most this many CTAs (0: one per SM, the resident limit).
template <int MAXS>
int launch(const ecf8_stream* streams, int n, cudaStream_t stream, bool overlap, int max_ctas) {
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
    B.mul = Mul{8u, 4u, 1u, 0u};
    DeviceInfo info;
    int st = device_info(&info);
    if (st != ECF8_OK) return st;
    long long grid = (long long)info.sms * info.blocks_per_sm;
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    if (grid > total) grid = total;
    if (!overlap) {
        decode_kernel<MAXS><<<(unsigned)grid, kThreads, sizeof(Smem), stream>>>(B);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e);
        return ECF8_OK;
    }
    // Programmatic dependent launch: the grid may begin once the previous
    // kernel on the stream has let dependents start (or has finished).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, decode_kernel<MAXS>, B);
    if (e != cudaSuccess) return cuda_fail(e);
    return ECF8_OK;
}

int decode_batch(const ecf8_stream* streams, int n_streams, int threads_per_block, int bytes_per_thread,
                 bool overlap, int max_ctas, void* cuda_stream) {
    int st = check_format(threads_per_block, bytes_per_thread);
    if (st != ECF8_OK) return st;
    if (n_streams < 0 || (n_streams > 0 && !streams)) return ECF8_ERR_INVALID_ARGUMENT;
    // Validate everything before launching anything.
    for (int i = 0; i < n_streams; ++i) {
        DevStream d;
        st = make_stream(streams[i], &d);
        if (st != ECF8_OK) return st;
    }
    for (int i = 0; i < n_streams; i += ECF8_MAX_BATCH) {
        const int n = n_streams - i < ECF8_MAX_BATCH ? n_streams - i : ECF8_MAX_BATCH;
        st = launch<ECF8_MAX_BATCH>(streams + i, n, (cudaStream_t)cuda_stream, overlap, max_ctas);
        if (st != ECF8_OK) return st;
    }
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
    s.table = nullptr;
    return ecf8::launch<1>(&s, 1, (cudaStream_t)cuda_stream, false, 0);
}

int ecf8_decode_batch(const ecf8_stream* streams, int n_streams, int threads_per_block,
                      int bytes_per_thread, void* cuda_stream) {
    return ecf8::decode_batch(streams, n_streams, threads_per_block, bytes_per_thread, false, 0, cuda_stream);
}

int ecf8_decode_batch_flags(const ecf8_stream* streams, int n_streams, int threads_per_block,
                            int bytes_per_thread, uint32_t flags, void* cuda_stream) {
    if (flags & ~((uint32_t)ECF8_DECODE_OVERLAP_PREVIOUS | ECF8_DECODE_CTAS(0xffffu)))
        return ECF8_ERR_INVALID_ARGUMENT;
    const int max_ctas = (int)(flags >> ECF8_DECODE_CTAS_SHIFT);
    return ecf8::decode_batch(streams, n_streams, threads_per_block, bytes_per_thread,
                              (flags & ECF8_DECODE_OVERLAP_PREVIOUS) != 0, max_ctas, cuda_stream);
}

int ecf8_build_table(const uint8_t* luts, int n_luts, uint32_t* table, void* cuda_stream) {
    if (n_luts < 2 || n_luts > ECF8_MAX_LUTS || !luts || !table) return ECF8_ERR_INVALID_ARGUMENT;
    if (!ecf8::aligned(table, 16)) return ECF8_ERR_INVALID_ARGUMENT;
    ecf8::DeviceInfo info;
    int st = ecf8::device_info(&info);
    if (st != ECF8_OK) return st;
    ecf8::build_table_kernel<<<1, ecf8::kTableThreads, sizeof(ecf8::TableSmem), (cudaStream_t)cuda_stream>>>(
        luts, n_luts, table);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return ecf8::cuda_fail(e);
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
