/* TEST INFRASTRUCTURE — ORACLE ONLY (see oracle.h). Plain C, single source file.
 * Every sort below is made stable by breaking ties on the original position, so the results
 * are fully specified by the comments that cite the reference. */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp64 SpMM (src/main.cpp:202-207) ------------------------------------------------------ */
typedef struct {
    const int32_t *row_ptr, *col;
    const float *val, *B;
    int32_t O, r0, r1;
    double *out, *abs_out;
} spmm_job;

static void spmm_rows(const spmm_job* j) {
    for (int32_t r = j->r0; r < j->r1; ++r) {
        double* o = j->out + (size_t)r * j->O;
        double* a = j->abs_out ? j->abs_out + (size_t)r * j->O : NULL;
        for (int32_t k = 0; k < j->O; ++k) o[k] = 0.0;
        if (a)
            for (int32_t k = 0; k < j->O; ++k) a[k] = 0.0;
        for (int32_t p = j->row_ptr[r]; p < j->row_ptr[r + 1]; ++p) {
            const double v = (double)j->val[p];
            const float* b = j->B + (size_t)j->col[p] * j->O;
            for (int32_t k = 0; k < j->O; ++k) {
                o[k] += v * b[k];
                if (a) a[k] += fabs(v * b[k]);
            }
        }
    }
}

static void* spmm_thread(void* arg) {
    spmm_rows((const spmm_job*)arg);
    return NULL;
}

void oracle_spmm_fp64(int32_t M, const int32_t* row_ptr, const int32_t* col, const float* val, const float* B,
                      int32_t O, double* out, double* abs_out, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > M) nthreads = M > 0 ? M : 1;
    spmm_job* jobs = (spmm_job*)calloc((size_t)nthreads, sizeof(spmm_job));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int t = 0; t < nthreads; ++t) {
        spmm_job j = {row_ptr, col, val, B, O, (int32_t)((int64_t)M * t / nthreads),
                      (int32_t)((int64_t)M * (t + 1) / nthreads), out, abs_out};
        jobs[t] = j;
    }
    if (nthreads == 1) {
        spmm_rows(&jobs[0]);
    } else {
        for (int t = 0; t < nthreads; ++t) pthread_create(&th[t], NULL, spmm_thread, &jobs[t]);
        for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    }
    free(jobs);
    free(th);
}

void oracle_spmm_fp64_rows(const int32_t* row_ptr, const int32_t* col, const float* val, const float* B, int32_t O,
                           const int32_t* rows, int32_t nrows, double* out, double* abs_out) {
    for (int32_t i = 0; i < nrows; ++i) {
        const int32_t r = rows[i];
        for (int32_t k = 0; k < O; ++k) {
            out[(size_t)i * O + k] = 0.0;
            if (abs_out) abs_out[(size_t)i * O + k] = 0.0;
        }
        for (int32_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            const double v = (double)val[p];
            const float* b = B + (size_t)col[p] * O;
            for (int32_t k = 0; k < O; ++k) {
                out[(size_t)i * O + k] += v * b[k];
                if (abs_out) abs_out[(size_t)i * O + k] += fabs(v * b[k]);
            }
        }
    }
}

/* ---- half_scale (src/vcsr_mc.cu:14-22) ----------------------------------------------------- */
float oracle_half_scale(int64_t nnz, const float* val) {
    const float headroom = 60000.0f, min_normal = 6.103515625e-05f;
    float amax = 0.0f;
    for (int64_t i = 0; i < nnz; ++i) {
        const float a = fabsf(val[i]);
        if (a > amax) amax = a;
    }
    if (amax > headroom) return amax / headroom;
    if (amax > 0.0f && amax < min_normal) return amax / headroom;
    return 1.0f;
}

/* ---- VCSR build (src/vcsr_mc.cu:25-123, canonical ties) ------------------------------------ */
typedef struct {
    int32_t col, pos;
    float v;
} ent_t;

static int cmp_ent(const void* a, const void* b) {
    const ent_t *x = (const ent_t*)a, *y = (const ent_t*)b;
    if (x->col != y->col) return x->col < y->col ? -1 : 1;
    return x->pos < y->pos ? -1 : (x->pos > y->pos);
}

typedef struct {
    int32_t row, count;
    int64_t first; /* index into the segment-ordered entry arrays */
} pair_t;

static int cmp_pair_canonical(const void* a, const void* b) {
    const pair_t *x = (const pair_t*)a, *y = (const pair_t*)b;
    if (x->count != y->count) return x->count > y->count ? -1 : 1; /* count descending */
    return x->row < y->row ? -1 : (x->row > y->row);                /* then row ascending */
}

typedef struct {
    int32_t b, e;
    int64_t work;
    int32_t idx;
} item_t;

static int cmp_item(const void* a, const void* b) {
    const item_t *x = (const item_t*)a, *y = (const item_t*)b;
    if (x->work != y->work) return x->work > y->work ? -1 : 1; /* heaviest first */
    return x->idx < y->idx ? -1 : (x->idx > y->idx);           /* stable */
}

int oracle_build_vcsr(int32_t M, int32_t N, const int32_t* row_ptr, const int32_t* col, const float* val,
                      int fp32, int segw, oracle_vcsr* out) {
    memset(out, 0, sizeof(*out));
    if (segw != 16 && segw != 32 && segw != 48 && segw != 64) return 1;
    const int bundle = 16;
    const int64_t nnz = row_ptr[M];
    out->M = M;
    out->N = N;
    out->segw = segw;
    out->bundle = bundle;
    out->fp32 = fp32 ? 1 : 0;
    out->scale = fp32 ? 1.0f : oracle_half_scale(nnz, val);
    const float inv_scale = 1.0f / out->scale;
    const int32_t S = (N + segw - 1) / segw;
    out->num_segments = S;

    /* entries of each row ordered by (column, original position) */
    ent_t* ent = (ent_t*)malloc(sizeof(ent_t) * (size_t)(nnz > 0 ? nnz : 1));
    for (int32_t r = 0; r < M; ++r) {
        for (int32_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            ent[p].col = col[p];
            ent[p].pos = p;
            ent[p].v = val[p];
        }
        qsort(ent + row_ptr[r], (size_t)(row_ptr[r + 1] - row_ptr[r]), sizeof(ent_t), cmp_ent);
    }
    /* (segment, row) pairs, bucketed by segment, ascending row within a segment */
    int64_t* seg_off = (int64_t*)calloc((size_t)S + 1, sizeof(int64_t));
    for (int32_t r = 0; r < M; ++r) {
        int32_t prev = -1;
        for (int32_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            const int32_t sid = ent[p].col / segw;
            if (sid != prev) { seg_off[sid + 1]++; prev = sid; }
        }
    }
    for (int32_t s = 0; s < S; ++s) seg_off[s + 1] += seg_off[s];
    const int64_t npairs = seg_off[S];
    pair_t* pairs = (pair_t*)malloc(sizeof(pair_t) * (size_t)(npairs > 0 ? npairs : 1));
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)(S > 0 ? S : 1));
    for (int32_t s = 0; s < S; ++s) cur[s] = seg_off[s];
    for (int32_t r = 0; r < M; ++r) {
        int32_t p = row_ptr[r];
        while (p < row_ptr[r + 1]) {
            const int32_t sid = ent[p].col / segw;
            int32_t q = p + 1;
            while (q < row_ptr[r + 1] && ent[q].col / segw == sid) ++q;
            pair_t pr = {r, q - p, p};
            pairs[cur[sid]++] = pr;
            p = q;
        }
    }
    free(cur);
    /* order rows within each segment: count descending, row ascending */
    int64_t G = 0, slots = 0;
    for (int32_t s = 0; s < S; ++s) {
        pair_t* P = pairs + seg_off[s];
        const int64_t n = seg_off[s + 1] - seg_off[s];
        qsort(P, (size_t)n, sizeof(pair_t), cmp_pair_canonical);
        for (int64_t i = 0; i < n; i += bundle) {
            G++;
            slots += (int64_t)P[i].count * bundle; /* first row of a group is its deepest */
        }
    }
    out->n_groups = G;
    out->n_slots = slots;
    out->group_ptr = (int32_t*)malloc(sizeof(int32_t) * (size_t)(G + 1));
    out->group_depth = (int32_t*)malloc(sizeof(int32_t) * (size_t)(G > 0 ? G : 1));
    out->group_seg_base = (int32_t*)malloc(sizeof(int32_t) * (size_t)(G > 0 ? G : 1));
    out->group_rows = (int32_t*)malloc(sizeof(int32_t) * (size_t)(G > 0 ? 16 * G : 1));
    out->lcol = (int32_t*)malloc(sizeof(int32_t) * (size_t)(slots > 0 ? slots : 1));
    out->val = (float*)malloc(sizeof(float) * (size_t)(slots > 0 ? slots : 1));
    int64_t g = 0, slot = 0;
    for (int32_t s = 0; s < S; ++s) {
        const pair_t* P = pairs + seg_off[s];
        const int64_t n = seg_off[s + 1] - seg_off[s];
        for (int64_t i = 0; i < n; i += bundle, ++g) {
            const int32_t depth = P[i].count;
            out->group_ptr[g] = (int32_t)slot;
            out->group_depth[g] = depth;
            out->group_seg_base[g] = s * segw;
            for (int lane = 0; lane < bundle; ++lane)
                out->group_rows[g * 16 + lane] = i + lane < n ? P[i + lane].row : -1;
            for (int32_t d = 0; d < depth; ++d)
                for (int lane = 0; lane < bundle; ++lane, ++slot) {
                    const int64_t j = i + lane;
                    if (j < n && d < P[j].count) {
                        const ent_t* e = &ent[P[j].first + d];
                        out->lcol[slot] = e->col % segw;
                        out->val[slot] = e->v * inv_scale;
                    } else {
                        out->lcol[slot] = -1;
                        out->val[slot] = 0.0f;
                    }
                }
        }
    }
    out->group_ptr[G] = (int32_t)slots;
    free(pairs);
    free(seg_off);
    free(ent);

    /* work items: runs of <= chunk groups of one segment; heaviest first, stable */
    int64_t chunk = G / 4096;
    if (chunk > 32) chunk = 32;
    if (chunk < 1) chunk = 1;
    item_t* items = (item_t*)malloc(sizeof(item_t) * (size_t)(G > 0 ? G : 1));
    int32_t ni = 0;
    for (int64_t b = 0; b < G;) {
        int64_t e = b;
        while (e < G && e - b < chunk && out->group_seg_base[e] == out->group_seg_base[b]) ++e;
        item_t it = {(int32_t)b, (int32_t)e, (int64_t)out->group_ptr[e] - out->group_ptr[b], ni};
        items[ni++] = it;
        b = e;
    }
    qsort(items, (size_t)ni, sizeof(item_t), cmp_item);
    out->n_items = ni;
    out->item_gbeg = (int32_t*)malloc(sizeof(int32_t) * (size_t)(ni > 0 ? ni : 1));
    out->item_gend = (int32_t*)malloc(sizeof(int32_t) * (size_t)(ni > 0 ? ni : 1));
    for (int32_t i = 0; i < ni; ++i) {
        out->item_gbeg[i] = items[i].b;
        out->item_gend[i] = items[i].e;
    }
    free(items);
    return 0;
}

void oracle_vcsr_free(oracle_vcsr* v) {
    free(v->group_ptr);
    free(v->group_depth);
    free(v->group_seg_base);
    free(v->group_rows);
    free(v->lcol);
    free(v->val);
    free(v->item_gbeg);
    free(v->item_gend);
    memset(v, 0, sizeof(*v));
}

typedef struct {
    int32_t row, count;
    int64_t src_slot0; /* slot of depth 0 in the original layout */
    int32_t src_depth_stride;
} canon_t;

static int cmp_canon(const void* a, const void* b) {
    const canon_t *x = (const canon_t*)a, *y = (const canon_t*)b;
    if (x->count != y->count) return x->count > y->count ? -1 : 1;
    return x->row < y->row ? -1 : (x->row > y->row);
}

void oracle_canonicalize_vcsr(int64_t n_groups, int32_t segw, const int32_t* group_ptr, const int32_t* group_depth,
                              const int32_t* group_seg_base, int32_t* group_rows, int32_t* lcol, float* val) {
    (void)segw;
    int64_t g0 = 0;
    while (g0 < n_groups) {
        int64_t g1 = g0;
        while (g1 < n_groups && group_seg_base[g1] == group_seg_base[g0]) ++g1;
        /* positions of the segment [g0, g1) */
        const int64_t np = (g1 - g0) * 16;
        canon_t* pos = (canon_t*)malloc(sizeof(canon_t) * (size_t)np);
        int64_t n = 0;
        int64_t span0 = group_ptr[g0], span1 = group_ptr[g1];
        for (int64_t g = g0; g < g1; ++g)
            for (int lane = 0; lane < 16; ++lane) {
                const int32_t row = group_rows[g * 16 + lane];
                if (row < 0) continue;
                int32_t cnt = 0;
                while (cnt < group_depth[g] && lcol[group_ptr[g] + (int64_t)cnt * 16 + lane] >= 0) ++cnt;
                canon_t c = {row, cnt, group_ptr[g] + lane, 16};
                pos[n++] = c;
            }
        qsort(pos, (size_t)n, sizeof(canon_t), cmp_canon);
        /* snapshot the segment's slots, then rewrite */
        const int64_t ns = span1 - span0;
        int32_t* lc = (int32_t*)malloc(sizeof(int32_t) * (size_t)(ns > 0 ? ns : 1));
        float* vv = (float*)malloc(sizeof(float) * (size_t)(ns > 0 ? ns : 1));
        memcpy(lc, lcol + span0, sizeof(int32_t) * (size_t)ns);
        memcpy(vv, val + span0, sizeof(float) * (size_t)ns);
        int64_t k = 0;
        for (int64_t g = g0; g < g1; ++g)
            for (int lane = 0; lane < 16; ++lane) {
                if (group_rows[g * 16 + lane] < 0) continue;
                const canon_t* c = &pos[k++];
                group_rows[g * 16 + lane] = c->row;
                for (int32_t d = 0; d < group_depth[g]; ++d) {
                    const int64_t dst = group_ptr[g] + (int64_t)d * 16 + lane;
                    if (d < c->count) {
                        const int64_t src = c->src_slot0 + (int64_t)d * c->src_depth_stride - span0;
                        lcol[dst] = lc[src];
                        val[dst] = vv[src];
                    } else {
                        lcol[dst] = -1;
                        val[dst] = 0.0f;
                    }
                }
            }
        free(lc);
        free(vv);
        free(pos);
        g0 = g1;
    }
}

/* ---- RCM (include/reorder.hpp:17-77) ------------------------------------------------------ */
typedef struct {
    int32_t key, pos, v;
} kv_t;

static int cmp_kv(const void* a, const void* b) {
    const kv_t *x = (const kv_t*)a, *y = (const kv_t*)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->pos < y->pos ? -1 : (x->pos > y->pos);
}

static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return x < y ? -1 : (x > y);
}

void oracle_rcm_column_order(int32_t M, int32_t N, const int32_t* row_ptr, const int32_t* col, int32_t* position) {
    const int32_t n = N;
    int64_t* head = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
    for (int32_t r = 0; r < M; ++r)
        for (int32_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            if (r < n) head[r + 1]++;
            head[col[p] + 1]++;
        }
    for (int32_t i = 0; i < n; ++i) head[i + 1] += head[i];
    int32_t* adj = (int32_t*)malloc(sizeof(int32_t) * (size_t)(head[n] > 0 ? head[n] : 1));
    int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    for (int32_t i = 0; i < n; ++i) fill[i] = head[i];
    for (int32_t r = 0; r < M; ++r)
        for (int32_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            const int32_t c = col[p];
            if (r < n) adj[fill[r]++] = c;
            adj[fill[c]++] = r < n ? r : c;
        }
    int32_t* degree = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    for (int32_t i = 0; i < n; ++i) {
        int32_t* b = adj + head[i];
        const int64_t len = head[i + 1] - head[i];
        qsort(b, (size_t)len, sizeof(int32_t), cmp_i32);
        int64_t u = 0;
        for (int64_t k = 0; k < len; ++k)
            if (u == 0 || b[k] != b[u - 1]) b[u++] = b[k];
        degree[i] = (int32_t)u;
    }
    kv_t* roots = (kv_t*)malloc(sizeof(kv_t) * (size_t)(n > 0 ? n : 1));
    for (int32_t i = 0; i < n; ++i) { roots[i].key = degree[i]; roots[i].pos = i; roots[i].v = i; }
    qsort(roots, (size_t)n, sizeof(kv_t), cmp_kv);
    char* seen = (char*)calloc((size_t)n + 1, 1);
    int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    kv_t* fresh = (kv_t*)malloc(sizeof(kv_t) * (size_t)(n > 0 ? n : 1));
    int64_t tail = 0;
    for (int32_t ri = 0; ri < n; ++ri) {
        const int32_t root = roots[ri].v;
        if (seen[root]) continue;
        seen[root] = 1;
        int64_t headq = tail;
        order[tail++] = root;
        while (headq < tail) {
            const int32_t v = order[headq++];
            int32_t nf = 0;
            for (int64_t k = head[v]; k < head[v] + degree[v]; ++k) {
                const int32_t u = adj[k];
                if (!seen[u]) {
                    seen[u] = 1;
                    fresh[nf].key = degree[u];
                    fresh[nf].pos = nf;
                    fresh[nf].v = u;
                    nf++;
                }
            }
            qsort(fresh, (size_t)nf, sizeof(kv_t), cmp_kv);
            for (int32_t k = 0; k < nf; ++k) order[tail++] = fresh[k].v;
        }
    }
    for (int32_t i = 0; i < n; ++i) position[order[n - 1 - i]] = i;
    free(head);
    free(adj);
    free(fill);
    free(degree);
    free(roots);
    free(seen);
    free(order);
    free(fresh);
}

void oracle_apply_column_permutation(int32_t M, int32_t N, const int32_t* row_ptr, int32_t* col, float* val,
                                     float* B, int32_t O, const int32_t* position) {
    ent_t* tmp = NULL;
    size_t cap = 0;
    for (int32_t r = 0; r < M; ++r) {
        const int32_t s = row_ptr[r], e = row_ptr[r + 1];
        if ((size_t)(e - s) > cap) {
            cap = (size_t)(e - s);
            tmp = (ent_t*)realloc(tmp, sizeof(ent_t) * cap);
        }
        for (int32_t p = s; p < e; ++p) {
            tmp[p - s].col = position[col[p]];
            tmp[p - s].pos = p;
            tmp[p - s].v = val[p];
        }
        qsort(tmp, (size_t)(e - s), sizeof(ent_t), cmp_ent);
        for (int32_t p = s; p < e; ++p) {
            col[p] = tmp[p - s].col;
            val[p] = tmp[p - s].v;
        }
    }
    free(tmp);
    if (!B) return;
    float* moved = (float*)malloc(sizeof(float) * (size_t)N * (size_t)O);
    for (int32_t old = 0; old < N; ++old)
        memcpy(moved + (size_t)position[old] * O, B + (size_t)old * O, sizeof(float) * (size_t)O);
    memcpy(B, moved, sizeof(float) * (size_t)N * (size_t)O);
    free(moved);
}
