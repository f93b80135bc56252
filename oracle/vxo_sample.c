/* Sampling restatement -- TEST INFRASTRUCTURE ONLY.
 *
 * Literal C restatement of the reference's greedy and nucleus sampling in
 * stdlib/ai/transformer.vx: argmax (1163-1177) and sample_top_p (1179-1260)
 * with the file's own series exponential _exp (36-80): temperature division,
 * max, exp of the shifted scores, sum in index order, normalisation, the
 * exchange sort of the indices by descending probability (swap whenever a
 * later entry is strictly larger than the one at the current position), the
 * cumulative cutoff at top_p, the LCG draw (1664525 * seed + 1013904223) mod
 * 2^31 in 128-bit integers like the interpreter's, and the renormalised scan.
 * Compiled with -ffp-contract=off: every f64 operation rounds on its own, as
 * in the interpreter.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "vxo.h"

/* _exp, stdlib/ai/transformer.vx:36-80 */
double vxo_vx_exp(double x) {
    if (x > 88.0) return 1.0e38;
    if (x < -88.0) return 0.0;
    const double ln2 = 0.6931471805599453;
    double k_f = x / ln2;
    int64_t k = k_f >= 0.0 ? (int64_t)(k_f + 0.5) : (int64_t)(k_f - 0.5); /* `as i128`: toward zero */
    double r = x - (double)k * ln2;
    double sum = 1.0, term = 1.0;
    for (int i = 1; i <= 20; i++) {
        term = term * r / (double)i;
        sum = sum + term;
    }
    double pow2 = 1.0;
    if (k >= 0) {
        for (int64_t j = 0; j < k; j++) pow2 = pow2 * 2.0;
    } else {
        for (int64_t j = 0; j < -k; j++) pow2 = pow2 / 2.0;
    }
    return sum * pow2;
}

/* argmax, stdlib/ai/transformer.vx:1163-1177 */
int64_t vxo_argmax(const double *logits, size_t n) {
    if (n == 0) return 0;
    int64_t best = 0;
    double bv = logits[0];
    for (size_t i = 1; i < n; i++)
        if (logits[i] > bv) {
            bv = logits[i];
            best = (int64_t)i;
        }
    return best;
}

/* the draw u of sample_top_p: state = (1664525 * seed + 1013904223) % 2^31
 * (truncated remainder of 128-bit integers), u = state / 2^31 */
double vxo_lcg_uniform(int64_t seed) {
    __int128 st = (__int128)1664525 * (__int128)seed + (__int128)1013904223;
    st = st % (__int128)2147483648LL;
    return (double)(int64_t)st / 2147483648.0;
}

/* sample_top_p, stdlib/ai/transformer.vx:1179-1260 */
int64_t vxo_sample_top_p(const double *logits, size_t n, double temperature, double top_p, int64_t seed) {
    if (n == 0) return 0;
    double *scaled = (double *)malloc(n * sizeof(double));
    double *probs = (double *)malloc(n * sizeof(double));
    int64_t *idx = (int64_t *)malloc(n * sizeof(int64_t));
    for (size_t i = 0; i < n; i++) scaled[i] = logits[i] / temperature;
    double mx = scaled[0];
    for (size_t i = 1; i < n; i++)
        if (scaled[i] > mx) mx = scaled[i];
    double psum = 0.0;
    for (size_t j = 0; j < n; j++) {
        double e = vxo_vx_exp(scaled[j] - mx);
        probs[j] = e;
        psum = psum + e;
    }
    for (size_t k = 0; k < n; k++) probs[k] = probs[k] / psum;
    for (size_t i = 0; i < n; i++) idx[i] = (int64_t)i;
    for (size_t a = 0; a + 1 < n; a++)
        for (size_t b = a + 1; b < n; b++)
            if (probs[idx[b]] > probs[idx[a]]) {
                int64_t t = idx[a];
                idx[a] = idx[b];
                idx[b] = t;
            }
    double cumsum = 0.0;
    size_t cutoff = n;
    for (size_t ci = 0; ci < n; ci++) {
        cumsum = cumsum + probs[idx[ci]];
        if (cumsum >= top_p) {
            cutoff = ci + 1;
            break;
        }
    }
    double u = vxo_lcg_uniform(seed);
    double renorm = 0.0;
    for (size_t ri = 0; ri < cutoff; ri++) renorm = renorm + probs[idx[ri]];
    double acc = 0.0;
    int64_t out = idx[0];
    for (size_t si = 0; si < cutoff; si++) {
        acc = acc + probs[idx[si]] / renorm;
        if (acc >= u) {
            out = idx[si];
            break;
        }
    }
    free(scaled);
    free(probs);
    free(idx);
    return out;
}
