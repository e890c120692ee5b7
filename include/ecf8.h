/*
 * ecf8.h -- C ABI of the B200 (sm_100a) ECF8 decode engine.
 *
 * An ECF8 "stream" is one compressed block of e4m3 weights in the on-disk
 * layout the reference compressor writes (scripts/compress.py:239-247,
 * 607-612 of zeyuyang8/ecf8):
 *
 *   luts                u8[n_luts][256]   two-level byte LUTs + code-length row
 *   encoded             u8[n_bytes]       MSB-first Huffman bitstream of exponents
 *   packed_other_4bits  u8[n_elements/2]  sign+mantissa nibbles, even element high
 *   output_positions    u64[...]          first element of every 4096-byte group,
 *                                         plus a trailing n_elements
 *   gaps                u8[...]           4-bit start offset of every 8-byte window
 *
 * All pointers are device pointers owned by the caller.  No entry point
 * allocates memory, synchronises the device or the stream, or keeps state
 * between calls other than per-device launch attributes computed once.
 * Every decode entry point is asynchronous on `cuda_stream` (a cudaStream_t;
 * NULL = the legacy default stream) and returns a status code; a non-zero
 * status means nothing was launched.
 *
 * A stream the reference compressor did not produce (corrupt LUTs, gaps or
 * output positions) yields unspecified bytes inside outputs[0, n_elements)
 * but never makes a kernel read or write outside the buffers described here.
 */
#ifndef ECF8_H_
#define ECF8_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ECF8_ABI_VERSION 8

/* Status codes. */
#define ECF8_OK 0
#define ECF8_ERR_INVALID_ARGUMENT 1 /* a size or pointer is inconsistent */
#define ECF8_ERR_UNSUPPORTED 2      /* threads_per_block / bytes_per_thread */
#define ECF8_ERR_CUDA 3             /* a CUDA runtime call failed */
#define ECF8_ERR_TOO_LARGE 4        /* above ECF8_NOALLOC_MAX_ELEMENTS */

/* Limits of the stream format the kernels accept. */
#define ECF8_BYTES_PER_THREAD 8    /* window size in bytes (decode.cu:5) */
#define ECF8_THREADS_PER_BLOCK 512 /* windows per group (compress.py:7) */
#define ECF8_MAX_LUTS 18           /* row 0 + 16 prefix rows + length row */
#define ECF8_MAX_BATCH 256         /* streams per ecf8_decode_batch launch */
#define ECF8_TABLE_BYTES 86544     /* prepared decode table (ecf8_build_table) */

/* One stream of a batched decode; field meaning as in ecf8_decode(). */
typedef struct ecf8_stream {
    const uint8_t* luts;
    int32_t n_luts;
    int32_t reserved0;
    const uint8_t* encoded;
    int64_t n_bytes;
    const uint8_t* packed_other_4bits;
    const uint64_t* output_positions;
    int64_t n_output_positions;
    const uint8_t* gaps;
    int64_t n_gap_bytes;
    uint8_t* outputs;
    int64_t n_elements;
    const uint32_t* table; /* ECF8_TABLE_BYTES from ecf8_build_table(), or NULL (derived in-kernel) */
} ecf8_stream;

/*
 * Decodes one stream into outputs[0, n_elements).
 *
 * Replaces the reference kernel launch `_decode(grid=(ceil(n_bytes/4096),),
 * block=(512,), shared_mem=..., args=[luts, encoded, packed_other_4bits,
 * output_positions, gaps, outputs, n_luts, n_bytes, n_elements])`
 * (dfloat/run/run.py:24-33,97-119; kernel signature dfloat/run/decode.cu:16-26):
 * the first nine arguments keep the reference kernel's order and meaning.
 * The reference takes the array lengths of output_positions and gaps from the
 * launch grid; here they are passed explicitly (n_output_positions entries,
 * n_gap_bytes bytes) so that a short array is read safely.
 * threads_per_block / bytes_per_thread are the stream format's parameters
 * (config.json "dfloat_config", compress.py:669-674); only 512 / 8 are
 * supported.  n_elements must be even (two nibbles per packed byte) and
 * output_positions 8-byte aligned; other pointers may have any alignment
 * (16-byte aligned outputs and 8-byte aligned encoded / packed_other_4bits
 * take the vector path).
 */
int ecf8_decode(const uint8_t* luts, const uint8_t* encoded,
                const uint8_t* packed_other_4bits,
                const uint64_t* output_positions, const uint8_t* gaps,
                uint8_t* outputs, int n_luts, int64_t n_bytes,
                int64_t n_elements, int64_t n_output_positions,
                int64_t n_gap_bytes, int threads_per_block,
                int bytes_per_thread, void* cuda_stream);

/*
 * Derives a stream's multi-symbol decode table (ECF8_TABLE_BYTES, 16-byte
 * aligned device memory) from its LUTs, asynchronously on cuda_stream:
 * 8192 64-bit entries, one per 13-bit stream prefix, each up to six whole
 * symbols with their bit and symbol counts; one 16-bit mask of symbol start
 * offsets per entry; a copy of the LUTs (18 rows, zero padded) and a 16-byte
 * header.  The table depends on the LUTs only, so it can be built once when a
 * stream is loaded and passed in ecf8_stream.table to every later decode.
 * Every decode checks the stored LUT copy against the stream's LUTs and
 * derives the table itself when they differ (or when no table is given), so
 * a table built from other LUTs costs time but never correctness.
 * Corresponds to the per-block set-up the reference loader does once
 * (dfloat/run/run.py:453-458, shared_mem_size).
 */
int ecf8_build_table(const uint8_t* luts, int n_luts, uint32_t* table,
                     void* cuda_stream);

/*
 * Decodes n_streams independent streams with one persistent launch.  Stands
 * in for a loop of reference `_decode` launches, one per block
 * (dfloat/run/run.py:87-119 runs one per hooked module), e.g. all experts a
 * GPU owns in one MoE layer.  streams[] is read on the host during the call;
 * n_streams may exceed ECF8_MAX_BATCH (several launches are issued).
 */
int ecf8_decode_batch(const ecf8_stream* streams, int n_streams,
                      int threads_per_block, int bytes_per_thread,
                      void* cuda_stream);

/*
 * ecf8_decode_batch with flags.  flags = 0 behaves exactly like
 * ecf8_decode_batch; other bits than the ones below are rejected
 * (ECF8_ERR_INVALID_ARGUMENT).  Neither option has a counterpart in the
 * reference (whose launches are plain stream-ordered kernels).
 *
 * ECF8_DECODE_OVERLAP_PREVIOUS: launches with programmatic dependent launch.
 * The decode may start while the previous kernel on cuda_stream is still
 * running: it reads its inputs (luts, encoded, packed_other_4bits,
 * output_positions, gaps, table) and builds its tables at once, and writes
 * its outputs only after that kernel has completed.  Back-to-back decodes
 * (one per layer) then overlap one launch's set-up with the previous one's
 * last groups.  The caller guarantees that no work still in flight on the
 * stream writes the inputs; work writing or reading the outputs is ordered
 * as without the flag.
 *
 * ECF8_DECODE_CTAS(n), n in 1..65535 (bits 31..16): launches at most n CTAs
 * instead of one per SM; every CTA still holds a whole SM's worth of shared
 * memory.  A decode issued ahead of use on a second CUDA stream then leaves
 * the other SMs to the kernels of the first.  The output is the same.
 */
#define ECF8_DECODE_OVERLAP_PREVIOUS 1u
#define ECF8_DECODE_CTAS_SHIFT 16
#define ECF8_DECODE_CTAS(n) ((uint32_t)(n) << ECF8_DECODE_CTAS_SHIFT)
int ecf8_decode_batch_flags(const ecf8_stream* streams, int n_streams,
                            int threads_per_block, int bytes_per_thread,
                            uint32_t flags, void* cuda_stream);

/*
 * GPU encoder, producing byte-identical buffers to the reference stream packer
 * dfloat/utils.py:373-499 for the given code table.  Two steps:
 *
 * ecf8_encode_plan: exponents u8[n] (values 0..15) on the device; code_bits[16]
 * (host) the code length of each symbol (0 = symbol absent).  workspace must
 * hold ecf8_encode_workspace_bytes(n) bytes of device memory.  Writes into
 * its last three u64 (device memory) the total bit count, the encoded byte
 * count and the number of output_positions entries the stream will have, and
 * into the u64 before them the number of invalid exponents: bytes above 15 or
 * symbols whose code length is 0.  The stream exists only when that count is
 * 0 (the reference packer fails on such input: dfloat/utils.py:408 looks the
 * symbol up in the code table).
 *
 * ecf8_encode_emit: same exponents / code table plus code values and the EOF
 * code; writes encoded (capacity >= round-up of n_bytes to 4 bytes), gaps
 * (n_gap_bytes = ceil(n_bytes/4096) * 256) and output_positions (the count the
 * plan reported).  The three output buffers are cleared by the call; when the
 * plan counted invalid exponents nothing else is written.
 */
int64_t ecf8_encode_workspace_bytes(int64_t n);
int ecf8_encode_plan(const uint8_t* exponents, int64_t n,
                     const uint8_t* code_bits, int eof_bits, void* workspace,
                     void* cuda_stream);
int ecf8_encode_emit(const uint8_t* exponents, int64_t n,
                     const uint8_t* code_bits, const uint32_t* code_values,
                     int eof_bits, uint32_t eof_value, const void* workspace,
                     uint8_t* encoded, int64_t n_bytes, int64_t encoded_capacity,
                     uint8_t* gaps, int64_t n_gap_bytes,
                     uint64_t* output_positions, int64_t n_output_positions,
                     void* cuda_stream);

/*
 * ecf8_encode_noalloc: the packer above in one call that allocates nothing.
 * It has no counterpart in the reference (whose packer runs in Python on the
 * host).  It is for callers that cannot hand the library extra device memory:
 * code running inside another framework that owns all device memory through
 * its own pool (a stray cudaMalloc can fail there, or fragment the pool), and
 * latency-sensitive loaders for which cudaMalloc's implicit device
 * synchronisation would stall other streams.  Such a caller passes only the
 * exponents, the code table and output buffers.
 *
 * Its working memory (per-chunk bit offsets) is a fixed array inside the
 * library, one per GPU that loads it, kept until the process exits, sized
 * for n <= ECF8_NOALLOC_MAX_ELEMENTS exponents (about 0.5 MB); larger n
 * returns ECF8_ERR_TOO_LARGE.  The first call on a device looks up that
 * array's device address; make the first call on each device before any
 * stream capture.  All calls share the array: calls whose work overlaps on
 * the GPU (different streams, or different host threads) race and must be
 * serialised by the caller.
 *
 * Outputs are cleared in full and must hold the longest stream the code
 * table allows for n symbols (L = the longest code length in code_bits):
 * encoded_capacity >= ceil(n*L/8) rounded up to 4, gaps_capacity >=
 * ceil(ceil(n*L/8)/4096)*256 bytes, output_positions_capacity >= that group
 * count + 2 entries.  sizes (3 u64, device) receives the total bit count, the
 * encoded byte count and the number of output_positions entries; the buffers
 * equal ecf8_encode_emit()'s for the same input up to those sizes (gaps up to
 * ceil(n_bytes/4096)*256 bytes).  An exponent above 15, or one whose symbol
 * has code length 0, makes sizes {0, 0, 0} and leaves the outputs cleared.
 * Asynchronous on cuda_stream.
 */
#define ECF8_NOALLOC_MAX_ELEMENTS 268435456LL
int ecf8_encode_noalloc(const uint8_t* exponents, int64_t n,
                        const uint8_t* code_bits, const uint32_t* code_values,
                        int eof_bits, uint32_t eof_value, uint8_t* encoded,
                        int64_t encoded_capacity, uint8_t* gaps,
                        int64_t gaps_capacity, uint64_t* output_positions,
                        int64_t output_positions_capacity, uint64_t* sizes,
                        void* cuda_stream);

/* Human-readable text for a status code. */
const char* ecf8_status_string(int status);

/* The CUDA error code behind the last ECF8_ERR_CUDA of this thread (0 if none). */
int ecf8_last_cuda_error(void);

/* ECF8_ABI_VERSION of the loaded library. */
int ecf8_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ECF8_H_ */
