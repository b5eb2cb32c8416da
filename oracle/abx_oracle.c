/*
 * abx_oracle.c — CPU restatement of the AB-Attention IBCS and SIP stages.
 *
 * ORACLE INFRASTRUCTURE. This file is test infrastructure: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, and only as
 * the checker. The shipped library never calls it.
 *
 * Each function follows one reference kernel, step for step, in scalar C with
 * IEEE float/double arithmetic:
 *   oracle_cluster <- cluster_queries_kernel  csrc/ibcs.cu:106-238
 *   oracle_pool    <- pool_keys_kernel        csrc/ibcs.cu:244-266
 *   oracle_lse     <- ibcs_lse_kernel         csrc/ibcs.cu:270-489
 *   oracle_mix     <- ibcs_scores_kernel      csrc/ibcs.cu:495-538
 *   oracle_sip     <- sip_kernel              csrc/sip.cu:33-167
 * Rounding points (bf16 centroids and pooled keys, bf16 scaled centroids, fp16
 * LSE) and summation orders are reproduced. Three things cannot be on a CPU:
 * the GPU build uses --use_fast_math (approximate exp2/log2/division), the
 * tensor-core dot product accumulates in its own order, and CUB's block
 * reduction/scan trees are restated below only as far as their documented
 * structure goes. So CPU-vs-GPU agreement is checked with tolerances, and the
 * bit-exact gate is GPU-vs-reference-kernel on the GPU box.
 *
 * Build: see oracle/Makefile (gcc -O2 -shared -fPIC, no -ffast-math).
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HEAD_DIM 128
#define QUERY_BLOCK 128
#define CENTROIDS 8
#define KV4 4
#define SIP_THREADS 256
#define SIP_BUCKET 4

/* ---- 16-bit float helpers (round to nearest even) ------------------------ */

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

static float round_f16(float f) { return (float)(_Float16)f; }

uint16_t oracle_f32_to_f16_bits(float f) {
    _Float16 h = (_Float16)f;
    uint16_t bits;
    memcpy(&bits, &h, 2);
    return bits;
}

/* ---- clustering ----------------------------------------------------------- */

/* Squared distance summed as the reference warp does: lane p folds dims
 * p, p+32, p+64, p+96 (fused multiply-add, as the fmad build contracts it), then
 * the xor-butterfly 16,8,4,2,1 as seen from lane 0 (csrc/ibcs.cu:61-67,143-156). */
static float block_distance(const float* row, const float* center) {
    float part[32];
    for (int p = 0; p < 32; ++p) {
        float d = 0.0f;
        for (int k = 0; k < 4; ++k) {
            const float delta = row[p + 32 * k] - center[p + 32 * k];
            d = fmaf(delta, delta, d);
        }
        part[p] = d;
    }
    for (int width = 16; width > 0; width >>= 1)
        for (int p = 0; p < width; ++p) part[p] = part[p] + part[p + width];
    return part[0];
}

/* Farthest-first 8-centre clustering of each 128-query block
 * (csrc/ibcs.cu:106-238). q: bf16 bits [bh, seq, 128]. Outputs: centroids bf16
 * bits [rows, 8, 128], populations [rows, 8], assignments [rows, 128] (-1 past
 * the end), and optionally the float quotient before bf16 rounding. */
void oracle_cluster(const uint16_t* q, int64_t bh, int64_t seq, uint16_t* centroids,
                    float* populations, int32_t* assignments, float* centroid_f32) {
    const int64_t qb = (seq + QUERY_BLOCK - 1) / QUERY_BLOCK;
    float block[QUERY_BLOCK][HEAD_DIM];
    float mean[HEAD_DIM];
    float min_distance[QUERY_BLOCK];
    int assign[QUERY_BLOCK];
    for (int64_t h = 0; h < bh; ++h) {
        for (int64_t r = 0; r < qb; ++r) {
            const int64_t row = h * qb + r;
            const int64_t token0 = r * QUERY_BLOCK;
            const int n = (int)((seq - token0) < QUERY_BLOCK ? (seq - token0) : QUERY_BLOCK);
            for (int i = 0; i < QUERY_BLOCK; ++i)
                for (int d = 0; d < HEAD_DIM; ++d)
                    block[i][d] = i < n ? bf16_to_f32(q[((h * seq) + token0 + i) * HEAD_DIM + d]) : 0.0f;
            for (int d = 0; d < HEAD_DIM; ++d) {
                float sum = 0.0f;
                for (int i = 0; i < n; ++i) sum += block[i][d];
                mean[d] = sum / (float)n;
            }
            /* first centre: farthest from the mean, ties to the lowest index */
            int center = 0;
            float best = -INFINITY;
            for (int i = 0; i < n; ++i) {
                const float dist = block_distance(block[i], mean);
                if (dist > best) { best = dist; center = i; }
            }
            for (int i = 0; i < n; ++i) { min_distance[i] = INFINITY; assign[i] = 0; }
            for (int slot = 0; slot < CENTROIDS; ++slot) {
                float c[HEAD_DIM];
                memcpy(c, block[center], sizeof(c));
                for (int i = 0; i < n; ++i) {
                    const float dist = block_distance(block[i], c);
                    if (dist < min_distance[i]) { min_distance[i] = dist; assign[i] = slot; }
                }
                if (slot + 1 < CENTROIDS) {
                    best = -INFINITY;
                    center = 0;
                    for (int i = 0; i < n; ++i)
                        if (min_distance[i] > best) { best = min_distance[i]; center = i; }
                }
            }
            int counts[CENTROIDS] = {0};
            for (int i = 0; i < n; ++i) counts[assign[i]]++;
            for (int s = 0; s < CENTROIDS; ++s) populations[row * CENTROIDS + s] = (float)counts[s];
            if (assignments)
                for (int i = 0; i < QUERY_BLOCK; ++i) assignments[row * QUERY_BLOCK + i] = i < n ? assign[i] : -1;
            for (int s = 0; s < CENTROIDS; ++s) {
                for (int d = 0; d < HEAD_DIM; ++d) {
                    float sum = 0.0f;
                    for (int i = 0; i < n; ++i)
                        if (assign[i] == s) sum += block[i][d];
                    const float value = counts[s] > 0 ? sum / (float)counts[s] : 0.0f;
                    centroids[(row * CENTROIDS + s) * HEAD_DIM + d] = f32_to_bf16(value);
                    if (centroid_f32) centroid_f32[(row * CENTROIDS + s) * HEAD_DIM + d] = value;
                }
            }
        }
    }
}

/* ---- key pooling (csrc/ibcs.cu:244-266) ----------------------------------- */

void oracle_pool(const uint16_t* k, int64_t bh, int64_t seq, uint16_t* pooled) {
    const int64_t blocks = bh * (seq / KV4);
    for (int64_t b = 0; b < blocks; ++b)
        for (int rep = 0; rep < 2; ++rep)
            for (int d = 0; d < HEAD_DIM; ++d) {
                const float a = bf16_to_f32(k[(b * KV4 + 2 * rep) * HEAD_DIM + d]);
                const float c = bf16_to_f32(k[(b * KV4 + 2 * rep + 1) * HEAD_DIM + d]);
                pooled[(b * 2 + rep) * HEAD_DIM + d] = f32_to_bf16(0.5f * (a + c));
            }
}

/* ---- centroid x key log-sum-exp (csrc/ibcs.cu:270-489) -------------------- */

static void accumulate_lse(float* maximum, float* denominator, float value) {
    const float next = fmaxf(*maximum, value);
    *denominator = fmaf(*denominator, exp2f(*maximum - next), exp2f(value - next));
    *maximum = next;
}

static float pair_lse(float left, float right) {
    const float maximum = fmaxf(left, right);
    return maximum + log2f(fmaxf(exp2f(left - maximum) + exp2f(right - maximum), 1.0e-20f));
}

static void combine_lse(float* maximum, float* denominator, float other_max, float other_den) {
    const float next = fmaxf(*maximum, other_max);
    *denominator = fmaf(*denominator, exp2f(*maximum - next), other_den * exp2f(other_max - next));
    *maximum = next;
}

/* centroids: bf16 bits [rows, 8, 128] (unscaled), pooled: bf16 bits [bh, F, 2, 128].
 * lse: fp16 bits [rows, 8, F]; lse_max / lse_den: [rows, 8]. The 128-term dot
 * product is evaluated in double and rounded once to float (the tensor core's
 * own accumulation order is not restated). */
void oracle_lse(const uint16_t* centroids, const uint16_t* pooled, int64_t bh, int64_t qb, int64_t F,
                float kappa, uint16_t* lse, float* lse_max, float* lse_den) {
    float c[HEAD_DIM];
    for (int64_t h = 0; h < bh; ++h) {
        for (int64_t r = 0; r < qb; ++r) {
            const int64_t row = h * qb + r;
            for (int s = 0; s < CENTROIDS; ++s) {
                for (int d = 0; d < HEAD_DIM; ++d)
                    c[d] = round_bf16(bf16_to_f32(centroids[(row * CENTROIDS + s) * HEAD_DIM + d]) * kappa);
                float maximum[4], denominator[4];
                for (int lane = 0; lane < 4; ++lane) { maximum[lane] = -FLT_MAX; denominator[lane] = 0.0f; }
                for (int64_t j = 0; j < F; ++j) {
                    float x[2];
                    for (int rep = 0; rep < 2; ++rep) {
                        const uint16_t* p = pooled + ((h * F + j) * 2 + rep) * HEAD_DIM;
                        double acc = 0.0;
                        for (int d = 0; d < HEAD_DIM; ++d) acc += (double)c[d] * (double)bf16_to_f32(p[d]);
                        x[rep] = (float)acc;
                    }
                    const float stored = round_f16(pair_lse(x[0] + 1.0f, x[1] + 1.0f));
                    lse[(row * CENTROIDS + s) * F + j] = oracle_f32_to_f16_bits(stored);
                    accumulate_lse(&maximum[j & 3], &denominator[j & 3], stored);
                }
                /* (c0 (+) c1) (+) (c2 (+) c3) */
                combine_lse(&maximum[0], &denominator[0], maximum[1], denominator[1]);
                combine_lse(&maximum[2], &denominator[2], maximum[3], denominator[3]);
                combine_lse(&maximum[0], &denominator[0], maximum[2], denominator[2]);
                lse_max[row * CENTROIDS + s] = maximum[0];
                lse_den[row * CENTROIDS + s] = denominator[0];
            }
        }
    }
}

/* ---- population-weighted mixture (csrc/ibcs.cu:495-538) ------------------- */

void oracle_mix(const uint16_t* lse, const float* populations, const float* lse_max, const float* lse_den,
                int64_t rows, int64_t F, float* scores) {
    for (int64_t row = 0; row < rows; ++row) {
        float total = 0.0f;
        for (int s = 0; s < CENTROIDS; ++s) total += populations[row * CENTROIDS + s];
        for (int64_t j = 0; j < F; ++j) {
            float score = 0.0f;
            for (int s = 0; s < CENTROIDS; ++s) {
                _Float16 h;
                memcpy(&h, &lse[(row * CENTROIDS + s) * F + j], 2);
                const float value = (float)h;
                const float probability = exp2f(value - lse_max[row * CENTROIDS + s]) / lse_den[row * CENTROIDS + s];
                score = fmaf(populations[row * CENTROIDS + s], probability, score);
            }
            scores[row * F + j] = score / total;
        }
    }
}

/* ---- SIP (csrc/sip.cu:33-167) --------------------------------------------- */

/* Sum of 256 per-thread partials in the shape of a block reduction over 8 warps:
 * each warp folds its 32 lanes pairwise (1,2,4,8,16), then the warp totals are
 * added in warp order. */
static double block_sum(const double* partial) {
    double warp_total[SIP_THREADS / 32];
    for (int w = 0; w < SIP_THREADS / 32; ++w) {
        double v[32];
        for (int l = 0; l < 32; ++l) v[l] = partial[w * 32 + l];
        for (int offset = 1; offset < 32; offset <<= 1)
            for (int l = 0; l + offset < 32; l += 2 * offset) v[l] = v[l] + v[l + offset];
        warp_total[w] = v[0];
    }
    double total = warp_total[0];
    for (int w = 1; w < SIP_THREADS / 32; ++w) total = total + warp_total[w];
    return total;
}

/* scores [rows, population], offsets [rows] -> ids / log_weights [rows, samples]. */
void oracle_sip(const float* scores, const float* offsets, int64_t rows, int population, int32_t* ids,
                float* log_weights, int samples) {
    const int buckets = (population + SIP_BUCKET - 1) / SIP_BUCKET;
    float* values = (float*)malloc(sizeof(float) * (size_t)population);
    double* prefix = (double*)malloc(sizeof(double) * (size_t)(buckets + 1));
    double partial[SIP_THREADS];
    for (int64_t row = 0; row < rows; ++row) {
        const float* input = scores + row * population;
        int32_t* out = ids + row * samples;
        float* logs = log_weights + row * samples;
        for (int j = 0; j < population; ++j) values[j] = fmaxf(input[j], 1e-30f);
        int certain = 0;
        double scale = 0.0;
        for (;;) {
            double maximum = 0.0;
            for (int t = 0; t < SIP_THREADS; ++t) {
                double local = 0.0;
                for (int j = t; j < population; j += SIP_THREADS)
                    if (values[j] > 0.f) {
                        const double v = fmax((double)values[j], 1e-30);
                        local += v;
                        maximum = fmax(maximum, v);
                    }
                partial[t] = local;
            }
            const double total = block_sum(partial);
            scale = (double)(samples - certain) / total;
            int added = 0;
            if (maximum * scale >= 1.0) {
                for (int j = 0; j < population; ++j)
                    if (values[j] > 0.f && fmax((double)values[j], 1e-30) * scale >= 1.0) {
                        values[j] = -values[j];
                        ++added;
                    }
            }
            certain += added;
            if (added == 0) break;
        }
        int last_residual = population - 1;
        while (last_residual >= 0 && values[last_residual] <= 0.) --last_residual;
        int slot = 0;
        for (int j = 0; j < population; ++j)
            if (values[j] < 0.f) { out[slot] = j; logs[slot] = 0.f; ++slot; }
        /* bucket prefix: contiguous per-thread chunks of whole buckets; the
         * exclusive scan of chunk masses is restated as a sequential sum. */
        const int chunk = ((buckets + SIP_THREADS - 1) / SIP_THREADS) * SIP_BUCKET;
        const int residuals = samples - certain;
        double carry = 0.0;
        for (int t = 0; t < SIP_THREADS; ++t) {
            const int begin = t * chunk;
            const int end = begin + chunk < population ? begin + chunk : population;
            double cumulative = carry;
            double chunk_mass = 0.0;
            for (int j = begin; j < end; ++j) chunk_mass += values[j] > 0.f ? (double)values[j] * scale : 0.;
            for (int j = begin; j < end; ++j) {
                if (j % SIP_BUCKET == 0) prefix[j / SIP_BUCKET] = j > last_residual ? residuals : cumulative;
                cumulative += values[j] > 0.f ? (double)values[j] * scale : 0.;
            }
            carry += chunk_mass;
        }
        prefix[buckets] = residuals;
        for (int k = 0; k < residuals; ++k) {
            const double threshold = (double)offsets[row] + k;
            int lower = 0, upper = buckets;
            while (lower < upper) {
                const int middle = (lower + upper + 1) / 2;
                if (prefix[middle] <= threshold) lower = middle;
                else upper = middle - 1;
            }
            const int bucket = lower < buckets - 1 ? lower : buckets - 1;
            double mass = prefix[bucket];
            int selected = last_residual;
            const int stop = (bucket + 1) * SIP_BUCKET < population ? (bucket + 1) * SIP_BUCKET : population;
            for (int j = bucket * SIP_BUCKET; j < stop; ++j) {
                if (values[j] <= 0.f) continue;
                selected = j;
                mass += (double)values[j] * scale;
                if (mass > threshold) break;
            }
            out[certain + k] = selected;
            logs[certain + k] = (float)(-log2(fmax((double)input[selected], 1e-30) * scale));
        }
    }
    free(values);
    free(prefix);
}
