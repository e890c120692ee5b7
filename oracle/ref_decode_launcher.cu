// ref_decode_launcher.cu -- TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference kernel dfloat/run/decode.cu of zeyuyang8/ecf8
// UNMODIFIED (it is #included from the reference checkout, whose path the
// Makefile passes as REF_DECODE_CU) and exposes one C launcher with the
// reference's launch geometry (dfloat/run/run.py:97-119).  Built only into
// oracle/_ref/; tests use it as a second, independent oracle on the GPU.
#include REF_DECODE_CU

extern "C" int ref_decode_launch(const void* luts, const void* encoded, const void* packed,
                                 const void* output_positions, const void* gaps, void* outputs,
                                 int n_luts, int n_bytes, int n_elements, unsigned grid,
                                 unsigned block, unsigned shared_mem, void* stream) {
    if (grid == 0) return 0;
    decode<<<grid, block, shared_mem, (cudaStream_t)stream>>>(
        (const uint8_t*)luts, (const uint8_t*)encoded, (const uint8_t*)packed,
        (const uint64_t*)output_positions, (const uint8_t*)gaps, (uint8_t*)outputs, n_luts, n_bytes,
        n_elements);
    return (int)cudaGetLastError();
}
