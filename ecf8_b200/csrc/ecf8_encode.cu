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
// three numbers.  `emit` recomputes each element's absolute bit offset and
// writes codes word by word: a thread owns 16 consecutive elements, writes the
// 32-bit words wholly inside its bit range with plain stores and ORs the two
// words it may share with its neighbours atomically.

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
constexpr long long kWindowBits = 8LL * ECF8_BYTES_PER_THREAD;          // 64
constexpr long long kGroupBits = kWindowBits * ECF8_THREADS_PER_BLOCK;  // 32768

struct CodeTable {
    uint32_t val[16];
    uint8_t bits[16];
    uint32_t eof_val;
    int eof_bits;
};

thread_local int g_last_cuda_error = 0;

__device__ __forceinline__ uint32_t block_sum(uint32_t v, uint32_t* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint32_t s = 0;
    if (threadIdx.x < 32) {
        s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0u;
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    return s;  // valid in thread 0
}

// Loads the 16 exponents of thread slot `i0` (clamped to n; absent = -1).
__device__ __forceinline__ void load16(const uint8_t* ex, long long n, long long i0, int sym[kPerThread]) {
    if (i0 + kPerThread <= n && ((reinterpret_cast<uintptr_t>(ex + i0) & 15) == 0)) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(ex + i0));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) sym[j] = (int)((w[j >> 2] >> (8 * (j & 3))) & 0xffu);
    } else {
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) sym[j] = (i0 + j < n) ? (int)__ldg(ex + i0 + j) : -1;
    }
}

// The code table in shared memory: lanes look up different symbols, which
// the kernel-parameter (constant) bank would serve one address at a time.
struct SmemTable {
    uint32_t val[16];
    uint32_t bits[16];
};

__device__ __forceinline__ void load_table(SmemTable& t, const CodeTable& T) {
    if (threadIdx.x < 16) {
        t.val[threadIdx.x] = T.val[threadIdx.x];
        t.bits[threadIdx.x] = T.bits[threadIdx.x];
    }
    __syncthreads();
}

__device__ __forceinline__ uint32_t sym_bits(const SmemTable& t, int s) {
    return s < 0 ? 0u : t.bits[s & 15];
}

// Code bits of symbol s (bits 16..0) plus 1 << 17 for an exponent the code
// table cannot encode: a byte above 15 or a symbol whose code length is 0.
// Such exponents encode as nothing (their masked length is 0), so every
// offset stays inside the planned stream; the plan counts them and emit
// writes nothing when the count is not 0.
__device__ __forceinline__ uint32_t sym_bits_and_invalid(const SmemTable& t, int s) {
    if (s < 0) return 0u;
    const uint32_t b = t.bits[s & 15];
    return b | ((b == 0u || s > 15) ? (1u << 17) : 0u);
}

constexpr int kInvalidShift = 32;  // chunk sums: code bits in the low half, invalid exponents in the high half

// Per-chunk code-length sums (low half) and invalid-exponent counts (high half).
__global__ void __launch_bounds__(kThreads) chunk_bits_kernel(const uint8_t* __restrict__ ex, long long n,
                                                              const __grid_constant__ CodeTable T,
                                                              unsigned long long* __restrict__ chunk) {
    __shared__ uint32_t red[kThreads / 32];
    __shared__ SmemTable t;
    load_table(t, T);
    const long long i0 = (long long)blockIdx.x * kChunk + (long long)threadIdx.x * kPerThread;
    int sym[kPerThread];
    load16(ex, n, i0, sym);
    // One reduction for both sums: a chunk has at most 4096 x 16 = 2^16 code
    // bits (bits 16..0) and 4096 invalid exponents (bits 29..17).
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) v += sym_bits_and_invalid(t, sym[j]);
    v = block_sum(v, red);
    if (threadIdx.x == 0)
        chunk[blockIdx.x] = (unsigned long long)(v & 0x1ffffu) | ((unsigned long long)(v >> 17) << kInvalidShift);
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
    if (threadIdx.x == 0) carry = invalid = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (long long b = 0; b < n_chunks; b += kScanThreads) {
        const long long i = b + threadIdx.x;
        const unsigned long long raw = i < n_chunks ? chunk[i] : 0ull;
        const unsigned long long x = raw & 0xffffffffull;
        if (raw >> kInvalidShift) atomicAdd(&invalid, raw >> kInvalidShift);
        unsigned long long v = x;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, v, o);
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
        const unsigned long long incl = v + (warp ? wsum[warp - 1] : 0ull);
        if (i < n_chunks) chunk[i] = c0 + incl - x;
        __syncthreads();
        if (threadIdx.x == kScanThreads - 1) carry = c0 + incl;
        __syncthreads();
    }
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

// ORs `v` (big-endian bit order) into stream word `w`.  Words are byte
// swapped into memory order.
__device__ __forceinline__ void put_word(uint32_t* enc32, long long w, uint32_t v, bool shared_word) {
    if (!v) return;
    if (shared_word)
        atomicOr(enc32 + w, bswap32(v));
    else
        enc32[w] = bswap32(v);
}

__device__ __forceinline__ void put_gap(uint32_t* gaps32, unsigned long long window, uint32_t gap) {
    // Window j's 4 bits sit in byte j/2, high nibble for even j (np.packbits order).
    const unsigned long long byte = window >> 1;
    const uint32_t nib = (window & 1) ? gap : (gap << 4);
    if (nib) atomicOr(gaps32 + (byte >> 2), nib << (8 * (byte & 3)));
}

__global__ void __launch_bounds__(kThreads) emit_kernel(const uint8_t* __restrict__ ex, long long n,
                                                        const __grid_constant__ CodeTable T,
                                                        const unsigned long long* __restrict__ chunk,
                                                        uint8_t* __restrict__ encoded, long long n_bytes,
                                                        uint32_t* __restrict__ gaps32,
                                                        uint64_t* __restrict__ op) {
    __shared__ uint32_t wsum[kThreads / 32];
    __shared__ SmemTable t;
    load_table(t, T);
    const long long c = blockIdx.x;
    const long long i0 = c * kChunk + (long long)threadIdx.x * kPerThread;
    int sym[kPerThread];
    load16(ex, n, i0, sym);
    uint32_t local = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) local += sym_bits(t, sym[j]);
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
    const unsigned long long total = chunk[gridDim.x];
    if (chunk[gridDim.x + 1]) return;  // the plan counted invalid exponents: no stream
    const unsigned long long b0 = chunk[c] + (v - local) + (warp ? wsum[warp - 1] : 0u);
    if (local == 0) return;

    // Start bit of the element before this thread's first one.
    unsigned long long prev_start;
    if (i0 == 0)
        prev_start = ~0ull;
    else
        prev_start = b0 - T.bits[__ldg(ex + i0 - 1) & 15];

    uint32_t* enc32 = reinterpret_cast<uint32_t*>(encoded);
    const long long first_word = (long long)(b0 >> 5);
    unsigned long long pos = b0;
    long long cur_w = first_word;
    uint32_t cur = 0;
    long long last_i = -1;
    unsigned long long last_start = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        if (sym[j] < 0) break;
        const uint32_t len = t.bits[sym[j] & 15];
        const uint32_t code = t.val[sym[j] & 15];
        const long long i = i0 + j;
        // window / group bookkeeping (utils.py:392-406)
        const unsigned long long ps = (j == 0) ? prev_start : last_start;
        if (i == 0 || (ps >> 6) != (pos >> 6)) put_gap(gaps32, pos >> 6, (uint32_t)(pos & 63));
        if (i == 0 || (ps / kGroupBits) != (pos / kGroupBits)) op[pos / kGroupBits] = (uint64_t)i;
        // place the code's bits [pos, pos + len) -- len <= 16, so at most two words
        const uint32_t off = (uint32_t)(pos & 31);
        const long long w = (long long)(pos >> 5);
        if (w != cur_w) {
            put_word(enc32, cur_w, cur, cur_w == first_word);
            cur_w = w;
            cur = 0;
        }
        if (off + len <= 32) {
            cur |= code << (32 - off - len);
        } else {
            const uint32_t spill = off + len - 32;
            cur |= code >> spill;
            put_word(enc32, cur_w, cur, cur_w == first_word);
            cur_w = w + 1;
            cur = code << (32 - spill);
        }
        last_start = pos;
        last_i = i;
        pos += len;
    }
    // The last word may be shared with the next thread.
    const bool is_last_thread = (last_i == n - 1);
    if (is_last_thread && (total % 8)) {
        // utils.py:439-459: complete the final byte with the EOF code's
        // leading bits, add the gap / output position of the end if it starts
        // a new window / group.
        const uint32_t r = (uint32_t)(total % 8);
        const uint32_t room = 8 - r;
        const uint32_t ebits = (uint32_t)T.eof_bits;
        const uint32_t tail = (r + ebits >= 8) ? (T.eof_val >> (ebits - room)) & ((1u << room) - 1u)
                                               : (T.eof_val << (room - ebits)) & ((1u << room) - 1u);
        const long long w = (long long)(total >> 5);
        const uint32_t boff = (uint32_t)(total & 31);  // first free bit in word w
        const uint32_t shifted = tail << (32 - boff - room);
        if (w != cur_w) {
            put_word(enc32, cur_w, cur, true);
            cur_w = w;
            cur = 0;
        }
        cur |= shifted;
        if ((last_start >> 6) != (total >> 6)) put_gap(gaps32, total >> 6, (uint32_t)(total & 63));
        if ((last_start / kGroupBits) != (total / kGroupBits)) op[total / kGroupBits] = (uint64_t)n;
    }
    put_word(enc32, cur_w, cur, true);
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
    if (chunks > 0) chunk_bits_kernel<<<(unsigned)chunks, kThreads, 0, s>>>(exponents, n, T, chunk);
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
    if (chunks > 0) chunk_bits_kernel<<<(unsigned)chunks, kThreads, 0, s>>>(exponents, n, T, chunk);
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
