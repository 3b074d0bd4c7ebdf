/*
 * Oracle (test infrastructure and the timed CPU baseline, never the product): the int32 accumulators of an int8
 * submanifold convolution on the host cores, the integer form of the reference's fallback operator
 * (promptmoge/_fallback/flex_gemm/_core.py:399-441 under the QAT fake quantisation of moge/model/modules/qat.py:40-115):
 *
 *     acc[o][n] = sum over taps v with nmap[o][v] >= 0, channels c:  q[nmap[o][v]][c] * w[n][v][c]
 *
 * Exact integer arithmetic (int8 x int8 products summed in int32; |acc| <= 27 * 256 * 127^2 < 2^31), so the result
 * does not depend on the order of the sums.  Output rows are split over OpenMP threads; within a row, 16 output
 * channels at a time accumulate pairs of input channels with 16-bit multiply-add (two int8 products per 32-bit lane).
 */
#include <immintrin.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* q [m_in][ci] int8, nmap [m][27] int32 (-1 = absent), w [co][27][ci] int8 -> acc [m][co] int32.  ci even, co a
 * multiple of 16.  Returns 0, or -1 when an argument or a neighbour index is out of range or memory runs out. */
int oracle_conv_acc(const int8_t* q, int64_t m_in, const int32_t* nmap, int64_t m, const int8_t* w, int ci, int co,
                    int32_t* acc) {
    if (!q || !nmap || !w || !acc || m < 0 || m_in < 0 || ci <= 0 || co <= 0 || ci > 4096 || co > 4096 || (ci & 1) ||
        (co & 15))
        return -1;
    const int cp_n = ci / 2;
    /* weights as [tap][ci / 2][co][2] int16: the two input channels of a pair side by side for each output */
    int16_t* wt = (int16_t*)aligned_alloc(64, ((size_t)27 * ci * co * sizeof(int16_t) + 63) / 64 * 64);
    if (!wt) return -1;
    for (int n = 0; n < co; ++n)
        for (int v = 0; v < 27; ++v)
            for (int c = 0; c < ci; ++c)
                wt[(((size_t)v * cp_n + c / 2) * co + n) * 2 + (c & 1)] = w[((size_t)n * 27 + v) * ci + c];
    int bad = 0;
    const int64_t chunk = 64;     /* rows per task: one tap's weights serve them all while they sit in cache */
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
    for (int64_t o0 = 0; o0 < m; o0 += chunk) {
        const int64_t o1 = o0 + chunk < m ? o0 + chunk : m;
        memset(acc + o0 * co, 0, (size_t)(o1 - o0) * co * sizeof(int32_t));
        for (int v = 0; v < 27; ++v) {
            const int16_t* wv = wt + (size_t)v * cp_n * co * 2;
            for (int64_t o = o0; o < o1; ++o) {
                const int32_t src = nmap[o * 27 + v];
                if (src < 0) continue;
                if (src >= m_in) {
                    bad = 1;
                    continue;
                }
                const int8_t* x = q + (int64_t)src * ci;
                for (int nb = 0; nb < co; nb += 16) {
                    int32_t* ar = acc + o * co + nb;
                    __m256i a0 = _mm256_loadu_si256((const __m256i*)ar);
                    __m256i a1 = _mm256_loadu_si256((const __m256i*)(ar + 8));
                    const int16_t* wb = wv + (size_t)nb * 2;
                    for (int cp = 0; cp < cp_n; ++cp) {
                        const uint32_t pair =
                            (uint16_t)(int16_t)x[2 * cp] | ((uint32_t)(uint16_t)(int16_t)x[2 * cp + 1] << 16);
                        const __m256i xp = _mm256_set1_epi32((int)pair);
                        const int16_t* wr = wb + (size_t)cp * co * 2;
                        a0 = _mm256_add_epi32(a0, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i*)wr), xp));
                        a1 = _mm256_add_epi32(a1, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i*)(wr + 16)), xp));
                    }
                    _mm256_storeu_si256((__m256i*)ar, a0);
                    _mm256_storeu_si256((__m256i*)(ar + 8), a1);
                }
            }
        }
    }
    free(wt);
    return bad ? -1 : 0;
}
