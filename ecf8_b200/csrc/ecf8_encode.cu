// ecf8_encode.cu -- GPU ECF8 stream packer (product compressor path).
//
// Produces, for a given code table, byte-identical buffers to the reference
// packer dfloat/utils.py:373-499 (`_encode_exponents_for_cuda`):
//   encoded           MSB-first concatenation of the exponent codes; when the
//                     bit count is not a multiple of 8 the last byte is
//                     completed with the leading bits of the EOF code
//                     (utils.py:439-459);
//   gaps              for every 64-bit window, the offset of the first code
//                     that starts in it, 4 bits per window, high nibble first,
//                     zero padded to ceil(n_bytes/4096)*512 windows
//                     (utils.py:392-400,475-494);
//   output_positions  for every 4096-byte group the index of the first
//                     element whose code starts in it, then n (utils.py:405,463).
//
// Two launches per stream.  `plan` sums code lengths per 4096-element chunk
// and scans the chunk sums (one CTA), so the host can size the outputs from
// three numbers.  `emit` recomputes each element's absolute bit offset; a
// thread owns 16 consecutive elements and ORs their codes and the gap
// nibbles of the windows they start into the chunk's stream words and gap
// words, assembled in shared memory.  The CTA then stores the chunk's words
// with coalesced plain stores, except the first and last stream and gap words,
// which it may share with the neighbouring chunks: those it ORs atomically
// into the zeroed outputs.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "ecf8.h"

namespace ecf8enc {
namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 16;
constexpr int kChunk = kThreads * kPerThread;  // elements per chunk (4096)
constexpr int kScanThreads = 1024;
constexpr int kScanPer = 8;  // chunk sums per scan thread and pass
constexpr long long kWindowBits = 8LL * ECF8_BYTES_PER_THREAD;          // 64
constexpr long long kGroupBits = kWindowBits * ECF8_THREADS_PER_BLOCK;  // 32768
constexpr int kMaxCodeBits = 16;
// Stream words (from the chunk's first bit rounded down to 512) and gap words
// (8 windows of 64 bits each) one chunk can touch.
constexpr int kChunkWords = (kChunk * kMaxCodeBits + 511) / 32 + 1;
constexpr int kChunkGapWords = kChunk * kMaxCodeBits / 512 + 1;

struct CodeTable {
    uint32_t val[16];
    uint8_t bits[16];
    uint32_t eof_val;
    int eof_bits;
};

thread_local int g_last_cuda_error = 0;

// The code table in shared memory: lanes look up different symbols, which
// the kernel-parameter (constant) bank would serve one address at a time.
struct SmemTable {
    uint32_t bits[16];
    uint32_t code[16];  // code value << 16 | code length
};

__device__ __forceinline__ void load_table(SmemTable& t, const CodeTable& T) {
    if (threadIdx.x < 16) {
        t.bits[threadIdx.x] = T.bits[threadIdx.x];
        t.code[threadIdx.x] = T.val[threadIdx.x] << 16 | T.bits[threadIdx.x];
    }
    __syncthreads();
}

// Code bits of exponent byte b (bits 16..0), or 1 << 17 for a byte the code
// table cannot encode: one above 15 or a symbol whose code length is 0.  Such
// exponents encode as nothing (their length counts 0), so every offset stays
// inside the planned stream; the plan counts them and emit writes nothing
// when the count is not 0.
__device__ __forceinline__ void load_bits_table(uint32_t* lenx, const CodeTable& T) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        const uint32_t bits = b < 16 ? T.bits[b] : 0u;
        lenx[b] = bits ? bits : (1u << 17);
    }
    __syncthreads();
}

constexpr int kInvalidShift = 32;  // chunk sums: code bits in the low half, invalid exponents in the high half

// Per-chunk code-length sums (low half) and invalid-exponent counts (high half).
// A CTA sums kSumChunks chunks, so each thread has that many 16-byte loads in
// flight at once.  One reduction serves both sums: a chunk has at most
// 4096 x 16 = 2^16 code bits (bits 16..0) and 4096 invalid exponents
// (bits 29..17).
constexpr int kSumChunks = 4;

__global__ void __launch_bounds__(kThreads) chunk_bits_kernel(const uint8_t* __restrict__ ex, long long n,
                                                              const __grid_constant__ CodeTable T,
                                                              unsigned long long* __restrict__ chunk,
                                                              long long n_chunks) {
    __shared__ uint32_t red[kSumChunks][kThreads / 32];
    __shared__ uint32_t lenx[256];
    load_bits_table(lenx, T);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long c0 = (long long)blockIdx.x * kSumChunks;
    uint4 raw[kSumChunks];
    bool vec[kSumChunks];
#pragma unroll
    for (int k = 0; k < kSumChunks; ++k) {
        const long long i0 = (c0 + k) * kChunk + (long long)threadIdx.x * kPerThread;
        vec[k] = i0 + kPerThread <= n && ((reinterpret_cast<uintptr_t>(ex + i0) & 15) == 0);
        raw[k] = vec[k] ? __ldg(reinterpret_cast<const uint4*>(ex + i0)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < kSumChunks; ++k) {
        const long long i0 = (c0 + k) * kChunk + (long long)threadIdx.x * kPerThread;
        uint32_t v = 0;
        if (vec[k]) {
            const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
            for (int j = 0; j < kPerThread; ++j) v += lenx[__byte_perm(w[j >> 2], 0u, 0x4440u + (j & 3))];
        } else {
            for (int j = 0; j < kPerThread; ++j)
                if (i0 + j < n) v += lenx[__ldg(ex + i0 + j)];
        }
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[k][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < kSumChunks && c0 + threadIdx.x < n_chunks) {
        uint32_t v = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) v += red[threadIdx.x][w];
        chunk[c0 + threadIdx.x] = (unsigned long long)(v & 0x1ffffu) | ((unsigned long long)(v >> 17) << kInvalidShift);
    }
}

// Exclusive scan of the chunk sums in place (chunk[c] becomes the first bit of
// chunk c) and the stream plan: plan[-1] invalid exponents, plan[0] total bits,
// plan[1] encoded bytes, plan[2] output_positions entries.
__global__ void __launch_bounds__(kScanThreads) scan_plan_kernel(const uint8_t* __restrict__ ex, long long n,
                                                                 const __grid_constant__ CodeTable T,
                                                                 unsigned long long* __restrict__ chunk,
                                                                 long long n_chunks,
                                                                 unsigned long long* __restrict__ plan) {
    __shared__ unsigned long long wsum[kScanThreads / 32];
    __shared__ unsigned long long carry;
    __shared__ unsigned long long invalid;
    // One pass's chunk sums, then their exclusive offsets within the pass
    // (at most 8192 x 2^16 = 2^29 bits): global memory is read and written
    // with consecutive threads on consecutive chunks.
    __shared__ __align__(16) uint32_t sv[kScanThreads * kScanPer];
    if (threadIdx.x == 0) carry = invalid = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long bad = 0;
    for (long long b = 0; b < n_chunks; b += (long long)kScanThreads * kScanPer) {
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            const long long i = b + k * kScanThreads + threadIdx.x;
            const unsigned long long raw = i < n_chunks ? chunk[i] : 0ull;
            sv[k * kScanThreads + threadIdx.x] = (uint32_t)raw;  // at most 2^16 code bits per chunk
            bad += raw >> kInvalidShift;
        }
        __syncthreads();
        // Thread t scans chunks b + 8t .. b + 8t + 7.
        uint4* mine = reinterpret_cast<uint4*>(sv + threadIdx.x * kScanPer);
        const uint4 p0 = mine[0], p1 = mine[1];
        const uint32_t xs[kScanPer] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        uint32_t x = 0;
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) x += xs[k];
        uint32_t v = x;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        if (lane == 31) wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            unsigned long long s = wsum[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            wsum[lane] = s;
        }
        __syncthreads();
        const unsigned long long c0 = carry;
        const uint32_t incl = v + (warp ? (uint32_t)wsum[warp - 1] : 0u);
        uint32_t run = incl - x, o[kScanPer];
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            o[k] = run;
            run += xs[k];
        }
        mine[0] = make_uint4(o[0], o[1], o[2], o[3]);
        mine[1] = make_uint4(o[4], o[5], o[6], o[7]);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kScanPer; ++k) {
            const long long i = b + k * kScanThreads + threadIdx.x;
            if (i < n_chunks) chunk[i] = c0 + sv[k * kScanThreads + threadIdx.x];
        }
        if (threadIdx.x == kScanThreads - 1) carry = c0 + incl;
        __syncthreads();
    }
    if (bad) atomicAdd(&invalid, bad);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long total = carry;
        chunk[n_chunks] = total;
        unsigned long long n_bytes = total / 8 + ((total % 8) ? 1 : 0);
        unsigned long long n_op = 1;  // utils.py:463 trailing entry
        if (n > 0) {
            const unsigned long long last_start = total - T.bits[__ldg(ex + n - 1) & 15];
            n_op += last_start / kGroupBits + 1;
            if ((total % 8) && total / kGroupBits > last_start / kGroupBits) n_op += 1;  // utils.py:444-445
        }
        plan[-1] = invalid;
        plan[0] = total;
        plan[1] = n_bytes;
        plan[2] = n_op;
    }
}

__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// Window j's 4 bits sit in byte j/2, high nibble for even j (np.packbits
// order); gap word j/8 holds bytes 4(j/8) .. 4(j/8)+3.  `q` is a code's
// start bit relative to a 512-bit-aligned origin, `gw` its gap word there.
__device__ __forceinline__ void put_gap(uint32_t* sg, uint32_t gw, uint32_t q) {
    const uint32_t window = q >> 6;  // parity and byte-in-word as for the absolute window
    const uint32_t gap = q & 63u;
    const uint32_t nib = (window & 1) ? gap : (gap << 4);
    if (nib) atomicOr(sg + gw, nib << (8 * ((window >> 1) & 3)));
}

// Stores words [0, count) of a chunk's shared-memory buffer at dst + first;
// the first and last word with atomicOr (the neighbouring chunks may own bits
// of them), the rest with plain stores.
__device__ __forceinline__ void store_chunk_words(uint32_t* dst, unsigned long long first, const uint32_t* src,
                                                  int count, bool swap) {
    for (int k = threadIdx.x; k < count; k += blockDim.x) {
        const uint32_t v = swap ? bswap32(src[k]) : src[k];
        if (k == 0 || k == count - 1) {
            if (v) atomicOr(dst + first + k, v);
        } else {
            dst[first + k] = v;
        }
    }
}

// Emits one thread's codes (its elements i0 .. i0 + 15 below n, the first
// starting at stream bit b0) into the chunk's shared stream words `sw` (word
// 0 = stream word A / 32) and gap words `sg` (word 0 = gap word A / 512).
// Positions are 32-bit: q = bit - (A - Ag), measured from the start of the
// 32768-bit group holding A (A is 512-aligned, Ag = A mod 32768), so one XOR
// of consecutive code starts tells a new window (>= 64) and a new group
// (>= 32768) (utils.py:392-406).  Codes shift into a 64-bit accumulator; each
// time one completes a 32-bit word, that word is ORed into `sw` (the first
// and last may hold the neighbouring threads' bits).  Output positions go
// straight to `op`: each is written by the one thread whose code starts its
// group.
__device__ __forceinline__ void emit_thread(uint32_t* sw, uint32_t* sg, unsigned long long A, uint32_t Ag,
                                            const SmemTable& t, const CodeTable& T, uint64_t* __restrict__ op,
                                            long long n, long long i0, const uint8_t* __restrict__ ex,
                                            const uint32_t (&w)[4], unsigned long long b0,
                                            unsigned long long total) {
    uint32_t q = (uint32_t)(b0 - A) + Ag;
    // Start of the element before this thread's first one; for element 0 of
    // the stream a value that differs from q in every bit (window 0 and
    // group 0 begin there).
    uint32_t prev = (i0 == 0) ? ~q : q - T.bits[__ldg(ex + i0 - 1) & 15];
    const uint32_t wofs = Ag >> 5, gofs = Ag >> 9;
    const unsigned long long group0 = A >> 15;
    uint32_t lo = 0, hi = 0;  // accumulator: the low (q mod 32) bits are the open word's
    const int m = (int)min((long long)kPerThread, n - i0);
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        if (j >= m) break;
        const uint32_t e = t.code[(w[j >> 2] >> (8 * (j & 3))) & 15u];
        const uint32_t len = e & 31u;
        const uint32_t x = q ^ prev;
        if (x >= 64u) {
            put_gap(sg, (q >> 9) - gofs, q);
            if (x >= 32768u) op[group0 + (q >> 15)] = (uint64_t)(i0 + j);
        }
        hi = __funnelshift_l(lo, hi, len);
        lo = (lo << len) | (e >> 16);
        const uint32_t end = q + len;
        if ((end ^ q) >= 32u) atomicOr(sw + (q >> 5) - wofs, __funnelshift_r(lo, hi, end));
        prev = q;
        q = end;
    }
    if (i0 + m == n && (total % 8)) {
        // utils.py:439-459: the last thread completes the final byte with the
        // EOF code's leading bits, and adds the gap / output position of the
        // end if it starts a new window / group.
        const uint32_t r = (uint32_t)(total % 8);
        const uint32_t room = 8 - r;
        const uint32_t ebits = (uint32_t)T.eof_bits;
        const uint32_t tail = (r + ebits >= 8) ? (T.eof_val >> (ebits - room)) & ((1u << room) - 1u)
                                               : (T.eof_val << (room - ebits)) & ((1u << room) - 1u);
        const uint32_t x = q ^ prev;
        if (x >= 64u) {
            put_gap(sg, (q >> 9) - gofs, q);
            if (x >= 32768u) op[group0 + (q >> 15)] = (uint64_t)n;
        }
        hi = __funnelshift_l(lo, hi, room);
        lo = (lo << room) | tail;
        const uint32_t end = q + room;
        if ((end ^ q) >= 32u) atomicOr(sw + (q >> 5) - wofs, __funnelshift_r(lo, hi, end));
        q = end;
    }
    if (q & 31u) atomicOr(sw + (q >> 5) - wofs, lo << (32 - (q & 31u)));
}

// Eight CTAs per SM (32 registers a thread): the CTAs' global loads and
// barriers overlap one another's emit work.
__global__ void __launch_bounds__(kThreads, 8) emit_kernel(const uint8_t* __restrict__ ex, long long n,
                                                        const __grid_constant__ CodeTable T,
                                                        const unsigned long long* __restrict__ chunk,
                                                        uint8_t* __restrict__ encoded, long long n_bytes,
                                                        uint32_t* __restrict__ gaps32,
                                                        uint64_t* __restrict__ op) {
    __shared__ uint32_t wsum[kThreads / 32];
    __shared__ SmemTable t;
    __shared__ uint32_t sw[kChunkWords];
    __shared__ uint32_t sg[kChunkGapWords];
    const long long c = blockIdx.x;
    const unsigned long long total = __ldg(chunk + gridDim.x), bad = __ldg(chunk + gridDim.x + 1);
    const unsigned long long cb0 = __ldg(chunk + c), cb1 = __ldg(chunk + c + 1);
    for (int k = threadIdx.x; k < kChunkWords; k += kThreads) sw[k] = 0u;
    for (int k = threadIdx.x; k < kChunkGapWords; k += kThreads) sg[k] = 0u;
    load_table(t, T);  // ends with a barrier
    const long long i0 = c * kChunk + (long long)threadIdx.x * kPerThread;
    uint32_t w[4];
    if (i0 + kPerThread <= n && ((reinterpret_cast<uintptr_t>(ex + i0) & 15) == 0)) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(ex + i0));
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t v = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) v |= (i0 + 4 * k + j < n ? (uint32_t)__ldg(ex + i0 + 4 * k + j) : 0u) << (8 * j);
            w[k] = v;
        }
    }
    uint32_t local = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j)
        local += (i0 + j < n) ? t.bits[(w[j >> 2] >> (8 * (j & 3))) & 15u] : 0u;
    // block exclusive scan of per-thread bit counts
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t v = local;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < kThreads / 32 ? wsum[lane] : 0u;
        for (int o = 1; o < kThreads / 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kThreads / 32) wsum[lane] = s;
    }
    __syncthreads();
    if (bad) return;  // the plan counted invalid exponents: no stream (uniform)
    const unsigned long long b0 = cb0 + (v - local) + (warp ? wsum[warp - 1] : 0u);
    // The chunk's codes start in bits [cb0, cb1); with the EOF completion of
    // the last byte (bits from `total`, in the word and gap word of bit
    // total - 1) they touch stream words [cb0/32, (cb1-1)/32] and gap words
    // [cb0/512, (cb1-1)/512].  The shared buffers start at A = cb0 rounded
    // down to 512 bits.
    const unsigned long long A = cb0 & ~511ull;
    if (local) emit_thread(sw, sg, A, (uint32_t)(A & 32767u), t, T, op, n, i0, ex, w, b0, total);
    __syncthreads();
    if (cb1 > cb0) {
        const unsigned long long w0 = cb0 >> 5;
        store_chunk_words(reinterpret_cast<uint32_t*>(encoded), w0, sw + (w0 - (A >> 5)),
                          (int)(((cb1 - 1) >> 5) - w0 + 1), true);
        store_chunk_words(gaps32, cb0 >> 9, sg, (int)(((cb1 - 1) >> 9) - (cb0 >> 9) + 1), false);
    }
    (void)n_bytes;
}

__global__ void op_tail_kernel(uint64_t* op, long long n_op, long long n) { op[n_op - 1] = (uint64_t)n; }

int cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return ECF8_ERR_CUDA;
}

int make_table(const uint8_t* code_bits, const uint32_t* code_values, int eof_bits, uint32_t eof_value,
               CodeTable* T) {
    if (!code_bits || eof_bits < 1 || eof_bits > 24) return ECF8_ERR_INVALID_ARGUMENT;
    for (int s = 0; s < 16; ++s) {
        if (code_bits[s] > 16) return ECF8_ERR_INVALID_ARGUMENT;
        T->bits[s] = code_bits[s];
        T->val[s] = code_values ? code_values[s] : 0u;
        if (code_values && code_bits[s] && (code_values[s] >> code_bits[s])) return ECF8_ERR_INVALID_ARGUMENT;
    }
    T->eof_bits = eof_bits;
    T->eof_val = eof_value;
    return ECF8_OK;
}

// --- No-allocation variant --------------------------------------------------
// Chunk bit offsets (+ total), the invalid-exponent count and the 3-entry
// plan for streams of up to kStaticMaxChunks chunks live in this file-scope
// array instead of a caller-provided workspace.  One copy per GPU that loads
// the library, held until the process exits.
constexpr long long kStaticMaxChunks = 65536;  // 65536 x 4096 = 268,435,456 elements
static_assert((long long)ECF8_NOALLOC_MAX_ELEMENTS == kStaticMaxChunks * kChunk, "limit mismatch");
static __device__ __align__(256) unsigned long long g_static_scratch[kStaticMaxChunks + 1 + 1 + 3];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
bool g_scratch_ready[kMaxDevices];
void* g_scratch_ptr[kMaxDevices];

// Writes the trailing output position from the plan the same launch sequence
// computed (nothing when the plan counted invalid exponents).
__global__ void op_tail_from_plan_kernel(uint64_t* op, const unsigned long long* plan, long long n) {
    if (plan[-1] == 0) op[plan[2] - 1] = (uint64_t)n;
}

// sizes = the plan, or {0, 0, 0} when it counted invalid exponents.
__global__ void copy_plan_kernel(uint64_t* sizes, const unsigned long long* plan) {
    if (threadIdx.x < 3) sizes[threadIdx.x] = plan[-1] ? 0ull : plan[threadIdx.x];
}

}  // namespace
}  // namespace ecf8enc

extern "C" {

int64_t ecf8_encode_workspace_bytes(int64_t n) {
    if (n < 0) return -1;
    const int64_t chunks = (n + ecf8enc::kChunk - 1) / ecf8enc::kChunk;
    return (chunks + 1 + 1 + 3) * 8;  // chunk starts + total, invalid-exponent count, the 3-entry plan
}

int ecf8_encode_plan(const uint8_t* exponents, int64_t n, const uint8_t* code_bits, int eof_bits,
                     void* workspace, void* cuda_stream) {
    using namespace ecf8enc;
    CodeTable T;
    int st = make_table(code_bits, nullptr, eof_bits, 0, &T);
    if (st != ECF8_OK) return st;
    if (n < 0 || (n > 0 && !exponents) || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 7))
        return ECF8_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)cuda_stream;
    const long long chunks = (n + kChunk - 1) / kChunk;
    unsigned long long* chunk = reinterpret_cast<unsigned long long*>(workspace);
    unsigned long long* plan = chunk + chunks + 2;
    if (chunks > 0x7fffffffLL) return ECF8_ERR_INVALID_ARGUMENT;
    if (chunks > 0)
        chunk_bits_kernel<<<(unsigned)((chunks + kSumChunks - 1) / kSumChunks), kThreads, 0, s>>>(exponents, n, T,
                                                                                             chunk, chunks);
    scan_plan_kernel<<<1, kScanThreads, 0, s>>>(exponents, n, T, chunk, chunks, plan);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return ECF8_OK;
}

int ecf8_encode_emit(const uint8_t* exponents, int64_t n, const uint8_t* code_bits,
                     const uint32_t* code_values, int eof_bits, uint32_t eof_value, const void* workspace,
                     uint8_t* encoded, int64_t n_bytes, int64_t encoded_capacity, uint8_t* gaps,
                     int64_t n_gap_bytes, uint64_t* output_positions, int64_t n_output_positions,
                     void* cuda_stream) {
    using namespace ecf8enc;
    CodeTable T;
    int st = make_table(code_bits, code_values, eof_bits, eof_value, &T);
    if (st != ECF8_OK) return st;
    if (!code_values || n < 0 || !workspace || n_output_positions < 1 || !output_positions)
        return ECF8_ERR_INVALID_ARGUMENT;
    const long long group_bytes = (long long)ECF8_THREADS_PER_BLOCK * ECF8_BYTES_PER_THREAD;
    const long long grid = (n_bytes + group_bytes - 1) / group_bytes;
    if (encoded_capacity < ((n_bytes + 3) & ~3LL) || n_gap_bytes != grid * (ECF8_THREADS_PER_BLOCK / 2))
        return ECF8_ERR_INVALID_ARGUMENT;
    if ((n_bytes > 0 && (!encoded || !gaps)) || (reinterpret_cast<uintptr_t>(encoded) & 3) ||
        (reinterpret_cast<uintptr_t>(gaps) & 3) || (reinterpret_cast<uintptr_t>(output_positions) & 7) ||
        (reinterpret_cast<uintptr_t>(workspace) & 7))
        return ECF8_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)cuda_stream;
    cudaError_t e = cudaSuccess;
    if (encoded_capacity > 0) e = cudaMemsetAsync(encoded, 0, (size_t)encoded_capacity, s);
    if (e == cudaSuccess && n_gap_bytes > 0) e = cudaMemsetAsync(gaps, 0, (size_t)n_gap_bytes, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(output_positions, 0, (size_t)n_output_positions * 8, s);
    if (e != cudaSuccess) return cuda_fail(e);
    const long long chunks = (n + kChunk - 1) / kChunk;
    const unsigned long long* chunk = reinterpret_cast<const unsigned long long*>(workspace);
    if (chunks > 0)
        emit_kernel<<<(unsigned)chunks, kThreads, 0, s>>>(exponents, n, T, chunk, encoded, n_bytes,
                                                          reinterpret_cast<uint32_t*>(gaps), output_positions);
    op_tail_kernel<<<1, 1, 0, s>>>(output_positions, n_output_positions, n);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return ECF8_OK;
}

// Single-call packer for callers that cannot allocate device memory; see
// include/ecf8.h.  Its scratch is the file-scope array g_static_scratch.
int ecf8_encode_noalloc(const uint8_t* exponents, int64_t n, const uint8_t* code_bits,
                        const uint32_t* code_values, int eof_bits, uint32_t eof_value, uint8_t* encoded,
                        int64_t encoded_capacity, uint8_t* gaps, int64_t gaps_capacity,
                        uint64_t* output_positions, int64_t output_positions_capacity, uint64_t* sizes,
                        void* cuda_stream) {
    using namespace ecf8enc;
    CodeTable T;
    int st = make_table(code_bits, code_values, eof_bits, eof_value, &T);
    if (st != ECF8_OK) return st;
    if (!code_values || n < 0 || (n > 0 && !exponents) || !sizes || !output_positions)
        return ECF8_ERR_INVALID_ARGUMENT;
    if (n > (int64_t)ECF8_NOALLOC_MAX_ELEMENTS) return ECF8_ERR_TOO_LARGE;
    // Capacities must cover the longest stream this code table can give for n
    // symbols (every symbol at the longest code length).
    int max_bits = 0;
    for (int k = 0; k < 16; ++k) max_bits = code_bits[k] > max_bits ? code_bits[k] : max_bits;
    const long long group_bytes = (long long)ECF8_THREADS_PER_BLOCK * ECF8_BYTES_PER_THREAD;
    const long long max_stream_bits = (long long)n * max_bits;
    const long long max_bytes = (max_stream_bits + 7) / 8;
    const long long max_groups = (max_bytes + group_bytes - 1) / group_bytes;
    if (encoded_capacity < ((max_bytes + 3) & ~3LL) || gaps_capacity < max_groups * (ECF8_THREADS_PER_BLOCK / 2) ||
        output_positions_capacity < max_groups + 2)
        return ECF8_ERR_INVALID_ARGUMENT;
    if ((max_bytes > 0 && (!encoded || !gaps)) || (reinterpret_cast<uintptr_t>(encoded) & 3) ||
        (reinterpret_cast<uintptr_t>(gaps) & 3) || (reinterpret_cast<uintptr_t>(output_positions) & 7) ||
        (reinterpret_cast<uintptr_t>(sizes) & 7))
        return ECF8_ERR_INVALID_ARGUMENT;
    // Set-up once per device, with that device current: the device address of
    // the scratch array (its name in host code is not a device pointer).
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return ECF8_ERR_UNSUPPORTED;
    // A failed lookup is not remembered: the next call on the device tries again.
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mutex);
        if (!g_scratch_ready[dev]) {
            void* ptr = nullptr;
            cudaError_t err = cudaGetSymbolAddress(&ptr, g_static_scratch);
            if (err != cudaSuccess) return cuda_fail(err);
            g_scratch_ptr[dev] = ptr;
            g_scratch_ready[dev] = true;
        }
        base = g_scratch_ptr[dev];
    }
    unsigned long long* chunk = static_cast<unsigned long long*>(base);
    const long long chunks = (n + kChunk - 1) / kChunk;
    unsigned long long* plan = chunk + chunks + 2;
    cudaStream_t s = (cudaStream_t)cuda_stream;
    // The scratch keeps the previous call's values; every entry this call
    // reads (chunk sums, their scan, the plan) is rewritten below before it is
    // read.  The outputs are cleared in full.
    if (encoded_capacity > 0) e = cudaMemsetAsync(encoded, 0, (size_t)encoded_capacity, s);
    if (e == cudaSuccess && gaps_capacity > 0) e = cudaMemsetAsync(gaps, 0, (size_t)gaps_capacity, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(output_positions, 0, (size_t)output_positions_capacity * 8, s);
    if (e != cudaSuccess) return cuda_fail(e);
    if (chunks > 0)
        chunk_bits_kernel<<<(unsigned)((chunks + kSumChunks - 1) / kSumChunks), kThreads, 0, s>>>(exponents, n, T,
                                                                                             chunk, chunks);
    scan_plan_kernel<<<1, kScanThreads, 0, s>>>(exponents, n, T, chunk, chunks, plan);
    if (chunks > 0)
        emit_kernel<<<(unsigned)chunks, kThreads, 0, s>>>(exponents, n, T, chunk, encoded, 0,
                                                          reinterpret_cast<uint32_t*>(gaps), output_positions);
    op_tail_from_plan_kernel<<<1, 1, 0, s>>>(output_positions, plan, n);
    copy_plan_kernel<<<1, 32, 0, s>>>(sizes, plan);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return ECF8_OK;
}

}  // extern "C"
