/*
 * ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C CPU restatement of the sparse NNUE feature-transformer math of
 * rgodha24/stockfish-trainer.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or as the timed CPU baseline.  The product path never
 * calls it.
 *
 * Every function names the reference lines it restates.  Summation orders are
 * kept identical to the reference so the forward and the weight gradient are
 * bit-exact:
 *   forward  : acc = bias; for k ascending: if idx != -1: acc += W[idx]
 *              (src/model/modules/feature_transformer/kernel.py:93-103)
 *   backward : stable sort of the flattened non-(-1) indices by feature,
 *              per feature acc = 0; for j in the segment (ascending position):
 *              acc += dOut[bid]; weight_grad[f] = weight_grad[f] + acc
 *              (kernel.py:108-138, 167-186); bias_grad += dOut.sum(0)
 *              (kernel.py:269).  The bias column sum is accumulated in double
 *              (torch's reduction order is not reproducible), so dB is only
 *              tolerance-equal.
 *   int16    : quantisation as src/model/quantize.py:83-89 (fp32 multiply,
 *              round half to even), accumulation as two's-complement int16
 *              (the engine submodule that runs it is absent from the reference).
 *
 * Built by oracle/build.py into oracle/_ref/liboracle_ft.so.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int oracle_threads(int nthreads) {
#ifdef _OPENMP
    return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

int oracle_max_threads(void) { return oracle_threads(0); }

/* kernel.py:89-103 -- one position at a time, bias first, then ascending k,
 * skipping -1.  Indices outside [0, T) other than -1 are skipped and counted
 * (the reference would read out of bounds); the count is returned. */
int64_t oracle_ft_forward(const int32_t *idx, int64_t B, int32_t K, const float *W,
                          int64_t T, int32_t C, const float *bias, float *out,
                          int nthreads) {
    int64_t bad = 0;
    int nt = oracle_threads(nthreads);
#pragma omp parallel for schedule(static) num_threads(nt) reduction(+ : bad)
    for (int64_t b = 0; b < B; ++b) {
        float *o = out + b * (int64_t)C;
        memcpy(o, bias, sizeof(float) * (size_t)C);
        const int32_t *row = idx + b * (int64_t)K;
        for (int32_t k = 0; k < K; ++k) {
            int32_t f = row[k];
            if (f == -1) continue;
            if (f < 0 || (int64_t)f >= T) { ++bad; continue; }
            const float *w = W + (int64_t)f * C;
            for (int32_t c = 0; c < C; ++c) o[c] += w[c];
        }
    }
    return bad;
}

/* kernel.py:108-138 -- flatten, drop -1, stable sort by feature, segments.
 * A counting sort scanned in flat order is stable, so it yields exactly the
 * permutation of torch.sort(stable=True).  Returns the number of unique
 * features U; sorted_bid has nnz entries, seg_* have U entries.  Indices
 * outside [-1, T) are dropped. */
int64_t oracle_ft_sorted_backward_inputs(const int32_t *idx, int64_t B, int32_t K,
                                         int64_t T, int32_t *sorted_bid,
                                         int32_t *seg_feat, int32_t *seg_count,
                                         int32_t *seg_start, int64_t *nnz_out) {
    int64_t *cnt = (int64_t *)calloc((size_t)T + 1, sizeof(int64_t));
    int64_t n = B * (int64_t)K;
    for (int64_t e = 0; e < n; ++e) {
        int32_t f = idx[e];
        if (f >= 0 && (int64_t)f < T) cnt[f + 1]++;
    }
    for (int64_t f = 0; f < T; ++f) cnt[f + 1] += cnt[f];
    int64_t nnz = cnt[T];
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (size_t)(T + 1));
    memcpy(cur, cnt, sizeof(int64_t) * (size_t)(T + 1));
    for (int64_t e = 0; e < n; ++e) {
        int32_t f = idx[e];
        if (f >= 0 && (int64_t)f < T) sorted_bid[cur[f]++] = (int32_t)(e / K);
    }
    int64_t u = 0;
    for (int64_t f = 0; f < T; ++f) {
        int64_t c = cnt[f + 1] - cnt[f];
        if (c == 0) continue;
        seg_feat[u] = (int32_t)f;
        seg_count[u] = (int32_t)c;
        seg_start[u] = (int32_t)cnt[f];
        ++u;
    }
    if (nnz_out) *nnz_out = nnz;
    free(cur);
    free(cnt);
    return u;
}

/* kernel.py:167-186 + :269 for ONE perspective, accumulating into caller
 * buffers exactly like the reference backward kernel: only touched rows of
 * dW are updated, dW[f] = dW[f] + acc with acc summed in ascending position
 * order.  dB += column sums (double accumulation). */
void oracle_ft_backward(const int32_t *idx, int64_t B, int32_t K, const float *dout,
                        int64_t T, int32_t C, float *dW, float *dB, int nthreads) {
    int64_t n = B * (int64_t)K;
    int32_t *sorted_bid = (int32_t *)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    int32_t *seg_feat = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1));
    int32_t *seg_count = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1));
    int32_t *seg_start = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1));
    int64_t nnz = 0;
    int64_t U = oracle_ft_sorted_backward_inputs(idx, B, K, T, sorted_bid, seg_feat,
                                                 seg_count, seg_start, &nnz);
    int nt = oracle_threads(nthreads);
#pragma omp parallel num_threads(nt)
    {
        float *acc = (float *)malloc(sizeof(float) * (size_t)C);
#pragma omp for schedule(dynamic, 64)
        for (int64_t u = 0; u < U; ++u) {
            for (int32_t c = 0; c < C; ++c) acc[c] = 0.0f;
            const int32_t *bids = sorted_bid + seg_start[u];
            for (int32_t j = 0; j < seg_count[u]; ++j) {
                const float *g = dout + (int64_t)bids[j] * C;
                for (int32_t c = 0; c < C; ++c) acc[c] += g[c];
            }
            float *w = dW + (int64_t)seg_feat[u] * C;
            for (int32_t c = 0; c < C; ++c) w[c] = w[c] + acc[c];
        }
        free(acc);
    }
    /* bias column sum */
    double *colsum = (double *)calloc((size_t)C, sizeof(double));
#pragma omp parallel num_threads(nt)
    {
        double *part = (double *)calloc((size_t)C, sizeof(double));
#pragma omp for schedule(static)
        for (int64_t b = 0; b < B; ++b) {
            const float *g = dout + b * (int64_t)C;
            for (int32_t c = 0; c < C; ++c) part[c] += g[c];
        }
#pragma omp critical
        for (int32_t c = 0; c < C; ++c) colsum[c] += part[c];
        free(part);
    }
    for (int32_t c = 0; c < C; ++c) dB[c] = dB[c] + (float)colsum[c];
    free(colsum);
    free(sorted_bid);
    free(seg_feat);
    free(seg_count);
    free(seg_start);
}

/* src/model/modules/features/halfka_v2_hm.py:100-134 -- training row (12
 * piece planes) -> export row (11 planes; both king planes share plane 10).
 * Valid for HalfKA feature indices produced by a legal-king position. */
int32_t oracle_halfka_export_row(int32_t i) {
    int32_t bucket = i / 768, plane = (i % 768) / 64, sq = i % 64;
    if (plane > 10) plane = 10;
    return bucket * 704 + plane * 64 + sq;
}

/* src/model/quantize.py:83-89: x.mul(scale).round() in fp32, half to even. */
void oracle_quantize_i16(const float *x, int64_t n, float scale, int16_t *q) {
    for (int64_t i = 0; i < n; ++i) q[i] = (int16_t)nearbyintf(x[i] * scale);
}
void oracle_quantize_i32(const float *x, int64_t n, float scale, int32_t *q) {
    for (int64_t i = 0; i < n; ++i) q[i] = (int32_t)nearbyintf(x[i] * scale);
}

/* Quantised FT forward (engine semantics; the engine is not in the
 * reference): acc[b, :L1] = bias_q + sum W_q[e(idx)] in int16 two's
 * complement, psqt[b, :] = sum Wpsqt_q[e(idx)] in int32.  map_training != 0
 * maps HalfKA training indices to export rows first. */
int64_t oracle_ft_quantized_forward(const int32_t *idx, int64_t B, int32_t K,
                                    const int16_t *Wq, const int32_t *Pq, int64_t Tq,
                                    int32_t L1, int32_t NP, const int16_t *bias_q,
                                    int map_training, int16_t *acc_out, int32_t *psqt_out,
                                    int nthreads) {
    int64_t bad = 0;
    int nt = oracle_threads(nthreads);
#pragma omp parallel for schedule(static) num_threads(nt) reduction(+ : bad)
    for (int64_t b = 0; b < B; ++b) {
        uint16_t *a = (uint16_t *)(acc_out + b * (int64_t)L1);
        int32_t *ps = psqt_out + b * (int64_t)NP;
        for (int32_t c = 0; c < L1; ++c) a[c] = (uint16_t)bias_q[c];
        for (int32_t c = 0; c < NP; ++c) ps[c] = 0;
        for (int32_t k = 0; k < K; ++k) {
            int32_t f = idx[b * (int64_t)K + k];
            if (f == -1) continue;
            if (map_training) {
                if (f < 0 || f >= 24576) { ++bad; continue; }
                f = oracle_halfka_export_row(f);
            }
            if (f < 0 || (int64_t)f >= Tq) { ++bad; continue; }
            const uint16_t *w = (const uint16_t *)(Wq + (int64_t)f * L1);
            for (int32_t c = 0; c < L1; ++c) a[c] = (uint16_t)(a[c] + w[c]);
            const int32_t *p = Pq + (int64_t)f * NP;
            for (int32_t c = 0; c < NP; ++c)
                ps[c] = (int32_t)((uint32_t)ps[c] + (uint32_t)p[c]);
        }
    }
    return bad;
}
