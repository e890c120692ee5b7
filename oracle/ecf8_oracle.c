/*
 * ecf8_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C restatement, for the host CPU, of the two reference routines that
 * define the ECF8 exponent-stream format:
 *
 *   1. the GPU decode kernel   dfloat/run/decode.cu:16-211   -> oracle_decode()
 *   2. the CPU stream packer   dfloat/utils.py:373-499       -> oracle_encode()
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library.  The product decode path lives in ecf8_b200/csrc and
 * never links against it.
 *
 * Deviations from the reference, all confined to bits that lie beyond the
 * real end of a stream (the EOF code and the padding after it), where the
 * reference itself is undefined:
 *   - bytes at or past n_bytes read as 0 (decode.cu:42-46 leaves those
 *     register bytes uninitialised);
 *   - a second-level LUT row index at or past n_luts reads as 0
 *     (decode.cu:88 would read past the end of `luts`);
 *   - a decoded code length of 0 advances by one bit (decode.cu:85-94 would
 *     spin forever); the number of such events is reported so tests know the
 *     reference kernel must not be run on that input.
 * On every stream the reference packer produces, none of these bits reach an
 * output byte below n_elements, so decoded bytes are identical.
 */
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_WINDOW_BYTES 8  /* decode.cu:5 BYTES_PER_THREAD */
#define ORACLE_LOOKAHEAD 2     /* decode.cu:6 BYTES_LOOK_AHEAD */

typedef struct {
    const uint8_t* luts;
    int n_luts;
    long long zero_len_events;
} lut_view;

/* decode.cu:86-88: first-level lookup by the top byte, second level by the
 * next byte when the first-level value is a row pointer (>= 240). */
static inline uint8_t lut_symbol(const lut_view* v, uint64_t buf) {
    uint8_t d = v->luts[buf >> 56];
    if (d >= 240) {
        int row = 256 - d;
        d = (row < v->n_luts) ? v->luts[256 * row + ((buf >> 48) & 0xff)] : 0;
    }
    return d;
}

/* decode.cu:91: code length from the last LUT row, indexed by symbol. */
static inline uint8_t lut_length(lut_view* v, uint8_t sym) {
    uint8_t len = v->luts[256 * (v->n_luts - 1) + sym];
    if (len == 0) {
        v->zero_len_events++;
        len = 1;
    }
    return len;
}

/* decode.cu:42-46 and 60-62: the 10-byte window of thread `gtid` and its gap. */
static void load_window(const uint8_t* enc, long long n_bytes, long long gtid,
                        uint8_t reg[ORACLE_WINDOW_BYTES + ORACLE_LOOKAHEAD]) {
    for (int i = 0; i < ORACLE_WINDOW_BYTES + ORACLE_LOOKAHEAD; i++) {
        long long pos = gtid * ORACLE_WINDOW_BYTES + i;
        reg[i] = pos < n_bytes ? enc[pos] : 0;
    }
}

static inline uint8_t load_gap(const uint8_t* gaps, long long gtid) {
    uint8_t b = gaps[gtid * 4 / 8];
    int bit_position = (int)(gtid * 4 % 8);
    return (uint8_t)((b >> (4 - bit_position)) & 0x0f);
}

static inline uint64_t window_be64(const uint8_t reg[]) {
    uint64_t w = 0;
    for (int i = 0; i < 8; i++) w = (w << 8) | reg[i];
    return w;
}

/* decode.cu:65-112 (pass 1): number of codes that start in bits [gap, 64). */
static uint32_t count_window(lut_view* v, const uint8_t reg[], uint8_t gap) {
    uint64_t buf = window_be64(reg) << gap;
    uint32_t free_bits = gap, count = 0;
    while (free_bits < 16) {
        uint8_t d = lut_symbol(v, buf);
        count++;
        uint8_t len = lut_length(v, d);
        buf <<= len;
        free_bits += len;
    }
    uint16_t la = (uint16_t)((reg[8] << 8) | reg[9]);
    buf |= (uint64_t)la << (free_bits - 16);
    free_bits -= 16;
    while (2 + free_bits / 8 < ORACLE_WINDOW_BYTES) {
        uint8_t d = lut_symbol(v, buf);
        count++;
        uint8_t len = lut_length(v, d);
        buf <<= len;
        free_bits += len;
    }
    return count;
}

/* decode.cu:174-176: merge exponent `e` with sign+mantissa nibble of element i. */
static inline uint8_t merge_byte(const uint8_t* packed, uint64_t i, uint8_t e) {
    uint8_t nib = (uint8_t)(packed[i / 2] << ((i % 2) * 4));
    return (uint8_t)((e << 3) | (nib & 0x80) | ((nib >> 4) & 0x7));
}

/* decode.cu:156-205 (pass 2): re-decode and place elements [start, end). */
static void emit_window(lut_view* v, const uint8_t reg[], uint8_t gap,
                        const uint8_t* packed, uint8_t* out, uint64_t start,
                        uint64_t end, uint64_t lo, uint64_t hi) {
    uint64_t buf = window_be64(reg) << gap;
    uint32_t free_bits = gap;
    uint64_t idx = start;
    while (free_bits < 16 && idx < end) {
        uint8_t d = lut_symbol(v, buf);
        if (idx >= lo && idx < hi) out[idx] = merge_byte(packed, idx, d);
        idx++;
        uint8_t len = lut_length(v, d);
        buf <<= len;
        free_bits += len;
    }
    /* The reference always performs the refill, even when pass 2 stopped
     * early; it has no effect on the elements already placed. */
    if (free_bits < 16) return;
    uint16_t la = (uint16_t)((reg[8] << 8) | reg[9]);
    buf |= (uint64_t)la << (free_bits - 16);
    free_bits -= 16;
    while (idx < end) {
        uint8_t d = lut_symbol(v, buf);
        if (idx >= lo && idx < hi) out[idx] = merge_byte(packed, idx, d);
        idx++;
        uint8_t len = lut_length(v, d);
        buf <<= len;
        free_bits += len;
    }
}

/*
 * Decodes one whole stream.  `output_positions` has n_output_positions
 * entries; group g reads entries g and g+1 (decode.cu:116,144-145).  An entry
 * the stream does not store (the reference would read past the array) is
 * taken as n_elements.  Bytes of `outputs` no group covers are left as they
 * are.  Groups run in parallel on up to `n_threads` OpenMP threads (<= 0: the
 * OpenMP default).  Returns the number of zero-length code events (0 on every
 * stream where the reference kernel terminates), or -1 on bad arguments.
 */
long long oracle_decode(const uint8_t* luts, int n_luts, const uint8_t* encoded,
                        long long n_bytes, const uint8_t* packed,
                        const uint64_t* output_positions,
                        long long n_output_positions, const uint8_t* gaps,
                        long long n_gap_bytes, uint8_t* outputs,
                        long long n_elements, int threads_per_block,
                        int n_threads) {
    if (n_luts < 2 || n_luts > 256 || threads_per_block <= 0 || n_bytes < 0 ||
        n_elements < 0 || n_output_positions < 1)
        return -1;
    long long bytes_per_group = (long long)threads_per_block * ORACLE_WINDOW_BYTES;
    long long grid = (n_bytes + bytes_per_group - 1) / bytes_per_group;
    if (n_gap_bytes * 2 < grid * threads_per_block) return -1;
    long long zero_len = 0;
#ifdef _OPENMP
    int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt) reduction(+ : zero_len)
#endif
    {
        lut_view v = {luts, n_luts, 0};
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (long long b = 0; b < grid; b++) {
            uint64_t seed = b < n_output_positions ? output_positions[b]
                                                   : (uint64_t)n_elements;
            uint64_t next = b + 1 < n_output_positions ? output_positions[b + 1]
                                                       : (uint64_t)n_elements;
            uint64_t hi = next < (uint64_t)n_elements ? next : (uint64_t)n_elements;
            /* pass 1 + exclusive scan seeded with output_positions[b] */
            uint64_t acc = seed;
            for (int t = 0; t < threads_per_block; t++) {
                long long gtid = b * threads_per_block + t;
                uint8_t reg[ORACLE_WINDOW_BYTES + ORACLE_LOOKAHEAD];
                load_window(encoded, n_bytes, gtid, reg);
                uint32_t c = count_window(&v, reg, load_gap(gaps, gtid));
                uint64_t start = acc;
                acc += c;
                /* pass 2 (decode.cu:151-152: end clamped by n_elements) */
                uint64_t end = acc < (uint64_t)n_elements ? acc : (uint64_t)n_elements;
                if (start < end)
                    emit_window(&v, reg, load_gap(gaps, gtid), packed, outputs,
                                start, end, seed, hi);
            }
        }
        zero_len += v.zero_len_events;
    }
    return zero_len;
}

/* ------------------------------------------------------------------------ */
/* Stream packer, restating dfloat/utils.py:373-499.                         */
/* ------------------------------------------------------------------------ */

/*
 * Sizes of the packer's outputs for `n` symbols: the encoded byte count, the
 * packed gap byte count and the number of output_positions entries.
 * code_bits[s] is the code length of symbol s (0..15; 0 = symbol absent).
 * Returns 0, or -1 when a symbol that occurs has no code.
 */
int oracle_encode_sizes(const uint8_t* sym, long long n, const uint8_t* code_bits,
                        int eof_bits, int bytes_per_thread, int threads_per_block,
                        long long* n_bytes, long long* n_gap_bytes,
                        long long* n_output_positions) {
    long long bits_per_thread = 8LL * bytes_per_thread;
    long long bits_per_block = bits_per_thread * threads_per_block;
    unsigned long long total = 0;
    long long n_op = 0, n_gaps = 0;
    (void)eof_bits;
    for (long long i = 0; i < n; i++) {
        uint8_t s = sym[i];
        if (s > 15 || code_bits[s] == 0) return -1;
        if ((long long)(total / bits_per_thread) + 1 > n_gaps) n_gaps++;
        if ((long long)(total / bits_per_block) + 1 > n_op) n_op++;
        total += code_bits[s];
    }
    long long nb = (long long)(total / 8);
    if (total % 8) {
        if ((long long)(total / bits_per_thread) + 1 > n_gaps) n_gaps++;
        if ((long long)(total / bits_per_block) + 1 > n_op) n_op++;
        nb++;
    }
    n_op++; /* utils.py:463 trailing total */
    long long grid = (nb + bits_per_block / 8 - 1) / (bits_per_block / 8);
    long long n_gap_entries = grid * threads_per_block;
    if (n_gaps > n_gap_entries) n_gap_entries = n_gaps; /* utils.py:477-478 */
    *n_bytes = nb;
    *n_gap_bytes = (n_gap_entries * 4 + 7) / 8;
    *n_output_positions = n_op;
    return 0;
}

/*
 * utils.py:373-499 for one stream.  code_val[s] / code_bits[s] is symbol s's
 * code (MSB-first), eof_val / eof_bits the EOF code.  Output arrays must have
 * the sizes oracle_encode_sizes() reports.  Returns 0.
 */
int oracle_encode(const uint8_t* sym, long long n, const uint8_t* code_bits,
                  const uint32_t* code_val, int eof_bits, uint32_t eof_val,
                  int bytes_per_thread, int threads_per_block, uint8_t* encoded,
                  uint8_t* gaps_packed, long long n_gap_bytes,
                  uint64_t* output_positions) {
    long long bits_per_thread = 8LL * bytes_per_thread;
    long long bits_per_block = bits_per_thread * threads_per_block;
    uint64_t buffer = 0; /* holds fewer than 8 + 16 pending bits */
    int size = 0;
    unsigned long long total = 0;
    long long n_gaps = 0, n_op = 0, n_enc = 0;
    memset(gaps_packed, 0, (size_t)n_gap_bytes);
#define PUT_GAP(gv)                                                        \
    do {                                                                   \
        uint8_t _g = (uint8_t)(gv);                                        \
        gaps_packed[n_gaps / 2] |= (uint8_t)((n_gaps % 2) ? _g : (_g << 4)); \
        n_gaps++;                                                          \
    } while (0)
    for (long long i = 0; i < n; i++) {
        /* utils.py:392-400 */
        if ((long long)(total / bits_per_thread) + 1 > n_gaps)
            PUT_GAP(total % bits_per_thread);
        /* utils.py:405-406 */
        if ((long long)(total / bits_per_block) + 1 > n_op)
            output_positions[n_op++] = (uint64_t)i;
        uint8_t s = sym[i];
        buffer = (buffer << code_bits[s]) | code_val[s];
        size += code_bits[s];
        total += code_bits[s];
        /* utils.py:422-432 */
        while (size >= 8) {
            encoded[n_enc++] = (uint8_t)(buffer >> (size - 8));
            size -= 8;
            buffer &= (size ? ((1ULL << size) - 1) : 0);
        }
    }
    /* utils.py:439-459 */
    if (size > 0) {
        if ((long long)(total / bits_per_thread) + 1 > n_gaps)
            PUT_GAP(total % bits_per_thread);
        if ((long long)(total / bits_per_block) + 1 > n_op)
            output_positions[n_op++] = (uint64_t)n;
        uint64_t b = (buffer << eof_bits) | eof_val;
        int sz = size + eof_bits;
        uint8_t byte;
        if (sz >= 8)
            byte = (uint8_t)(b >> (sz - 8));
        else
            byte = (uint8_t)(b << (8 - sz));
        encoded[n_enc++] = byte;
    }
    /* utils.py:463: trailing total; 475-483: remaining gap entries stay 0 */
    output_positions[n_op++] = (uint64_t)n;
#undef PUT_GAP
    return 0;
}

/* Splits e4m3 bytes into exponents and packed sign+mantissa nibbles exactly as
 * dfloat/utils.py:216-225 does; n must be even. */
void oracle_split(const uint8_t* w, long long n, uint8_t* exponents,
                  uint8_t* packed) {
    for (long long i = 0; i < n; i++) exponents[i] = (w[i] >> 3) & 0xF;
    for (long long j = 0; j < n / 2; j++) {
        uint8_t a = w[2 * j], b = w[2 * j + 1];
        uint8_t oa = (uint8_t)(((a >> 4) & 0x8) | (a & 0x7));
        uint8_t ob = (uint8_t)(((b >> 4) & 0x8) | (b & 0x7));
        packed[j] = (uint8_t)((oa << 4) | ob);
    }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
