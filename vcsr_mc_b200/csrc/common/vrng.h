/* Counter-based random numbers for the synthetic inputs (host C/C++ and CUDA device code).
 *
 * Every value is a pure function of (seed, stream, index), so host threads, GPU threads and
 * the numpy restatement in tests/golden/ all produce the same bits in any order.
 *   mix64   : the SplitMix64 output function (Steele, Lea & Flood, "Fast splittable
 *             pseudorandom number generators", OOPSLA 2014).
 *   key     : a stream key from (seed, stream id).
 *   at(k,i) : the i-th 64-bit draw of stream k = mix64(k + (i + 1) * golden gamma).
 *   u01     : top 53 bits as a double in [0, 1).
 *   sym     : a double in [-1, 1) rounded to float (U(-1,1)).
 */
#ifndef VCSRMC_VRNG_H
#define VCSRMC_VRNG_H
#include <stdint.h>

#if defined(__CUDACC__)
#define VRNG_FN static __host__ __device__ __forceinline__
#else
#define VRNG_FN static inline
#endif

#define VRNG_GAMMA 0x9E3779B97F4A7C15ULL

enum {
    VRNG_STREAM_ROWLEN = 1, /* row lengths (Poisson / Zipf draws)            */
    VRNG_STREAM_COLS = 2,   /* column choice per row                         */
    VRNG_STREAM_VALS = 3,   /* values of A, indexed by CSR position          */
    VRNG_STREAM_DENSE = 4,  /* dense B, indexed by row * cols + col          */
    VRNG_STREAM_RMAT = 5,   /* R-MAT quadrant choices                        */
    VRNG_STREAM_LINKS = 6   /* long-range links: column, value per link      */
};

VRNG_FN uint64_t vrng_mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ULL;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return z;
}
VRNG_FN uint64_t vrng_key(uint64_t seed, uint64_t stream) {
    return vrng_mix64(seed ^ vrng_mix64(stream * VRNG_GAMMA + 0xD1B54A32D192ED03ULL));
}
VRNG_FN uint64_t vrng_at(uint64_t key, uint64_t i) { return vrng_mix64(key + (i + 1) * VRNG_GAMMA); }
VRNG_FN double vrng_u01(uint64_t x) { return (double)(x >> 11) * (1.0 / 9007199254740992.0); }
VRNG_FN float vrng_sym(uint64_t x) {
    return (float)((double)(x >> 11) * (1.0 / 4503599627370496.0) - 1.0);
}

#endif
