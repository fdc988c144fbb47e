/*
 * TEST INFRASTRUCTURE ONLY — CPU restatement of the reference hot path (see vg_oracle.h).
 *
 * Build: gcc -O2 -march=x86-64-v3 -ffp-contract=off -fPIC -shared (oracle/Makefile). Contraction is
 * off so that every fused multiply-add below is the explicit fmaf() written here. The expressions
 * that decide the visited cells (walk distances, exit-face parameters, sample positions) use the
 * contraction nvcc applies to the reference's source, so that fp32 cell sequences agree bit for bit
 * with the CUDA kernels:
 *     a0*b0 + a1*b1 + a2*b2  ->  fma(a2, b2, fma(a0, b0, a1*b1))
 *     o + t*d               ->  fma(t, d, o)
 *     0.5f*(a + b) - c      ->  fma(0.5, a + b, -c)   (0.5 * x is exact)
 * Everything else (densities, colours, compositing) is plain fp32 with libm expf in place of the
 * kernels' __expf; those values are compared with tolerances.
 */
#include "vg_oracle.h"

#include <float.h>
#include <limits.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#define KINF 3.402823466e38f /* foam.cu:27 */
#define WALK_CAP 4096        /* foam.cu:29 */
#define MAX_CELLS 8192       /* foam.cu:30 */
#define MIN_WEIGHT 1e-7f     /* foam.cu:31 */
#define RECORD 8             /* foam.cu:274 */

static inline float dot3c(float a0, float a1, float a2, float b0, float b1, float b2) {
    return fmaf(a2, b2, fmaf(a0, b0, a1 * b1));
}

/* --------------------------------------------------------------------------------- threading */

typedef struct {
    int64_t n;
    int n_threads;
    void* ctx;
    void (*fn)(void* ctx, int64_t r);
    int tid;
} Job;

static void* job_main(void* arg) {
    Job* j = (Job*)arg;
    const int64_t chunk = (j->n + j->n_threads - 1) / j->n_threads;
    const int64_t a = chunk * j->tid, b = a + chunk < j->n ? a + chunk : j->n;
    for (int64_t r = a; r < b; ++r) j->fn(j->ctx, r);
    return NULL;
}

static void parallel_for(int64_t n, int n_threads, void* ctx, void (*fn)(void*, int64_t)) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_threads == 1 || n < 2) {
        for (int64_t r = 0; r < n; ++r) fn(ctx, r);
        return;
    }
    pthread_t th[256];
    Job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].n = n, jobs[t].n_threads = n_threads, jobs[t].ctx = ctx, jobs[t].fn = fn, jobs[t].tid = t;
        pthread_create(&th[t], NULL, job_main, &jobs[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* Gradient accumulation shared by the threads: striped spin locks per site. With one thread the
 * sums are deterministic. */
#define N_LOCKS 65536
static atomic_flag g_locks[N_LOCKS];
static int g_use_locks = 0;
static inline void lock_site(int k) {
    if (!g_use_locks) return;
    while (atomic_flag_test_and_set_explicit(&g_locks[(unsigned)k % N_LOCKS], memory_order_acquire)) {
    }
}
static inline void unlock_site(int k) {
    if (!g_use_locks) return;
    atomic_flag_clear_explicit(&g_locks[(unsigned)k % N_LOCKS], memory_order_release);
}

/* ------------------------------------------------------------------------------ field helpers */

typedef struct {
    const float* p;
    const int32_t* off;
    const int32_t* adj;
} Graph;

typedef struct {
    const float *raw, *dA, *cA, *sh;
    int deg;
} Field;

/* foam.cu:118-141 */
static void sh_basis(float x, float y, float z, int deg, float b[16]) {
    b[0] = 0.28209479177387814f;
    for (int i = 1; i < 16; ++i) b[i] = 0.f;
    if (deg < 1) return;
    b[1] = -0.4886025119029199f * y;
    b[2] = 0.4886025119029199f * z;
    b[3] = -0.4886025119029199f * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    b[4] = 1.0925484305920792f * x * y;
    b[5] = -1.0925484305920792f * y * z;
    b[6] = 0.31539156525252005f * (2.f * zz - xx - yy);
    b[7] = -1.0925484305920792f * x * z;
    b[8] = 0.5462742152960396f * (xx - yy);
    if (deg < 3) return;
    b[9] = -0.5900435899266435f * y * (3.f * xx - yy);
    b[10] = 2.890611442640554f * x * y * z;
    b[11] = -0.4570457994644658f * y * (4.f * zz - xx - yy);
    b[12] = 0.3731763325901154f * z * (2.f * zz - 3.f * xx - 3.f * yy);
    b[13] = -0.4570457994644658f * x * (4.f * zz - xx - yy);
    b[14] = 1.445305721320277f * z * (xx - yy);
    b[15] = -0.5900435899266435f * x * (xx - 3.f * yy);
}

/* foam.cu:143-153 */
static inline void sh_eval(const float* sh, int k, const float b[16], int nb, float c[3]) {
    const float* p = sh + 48 * (int64_t)k;
    c[0] = c[1] = c[2] = 0.5f;
    for (int j = 0; j < nb; ++j) {
        c[0] += b[j] * p[3 * j];
        c[1] += b[j] * p[3 * j + 1];
        c[2] += b[j] * p[3 * j + 2];
    }
}

/* foam.cu:101-105 */
static inline float maha(const float* A, int k, const float v[3]) {
    const float* a = A + 6 * (int64_t)k;
    return a[0] * v[0] * v[0] + a[3] * v[1] * v[1] + a[5] * v[2] * v[2] +
           2.f * (a[1] * v[0] * v[1] + a[2] * v[0] * v[2] + a[4] * v[1] * v[2]);
}

static inline void offset_to(const float* p, int k, const float x[3], float v[3]) {
    const int64_t k3 = 3 * (int64_t)k;
    v[0] = x[0] - p[k3], v[1] = x[1] - p[k3 + 1], v[2] = x[2] - p[k3 + 2];
}

static inline int neighbor(const Graph* g, int i, int e0, int e) { return e == 0 ? i : g->adj[e0 + e - 1]; }

/* Greedy walk to the nearest site of x, ties to the smaller index (foam.cu:163-181). */
static int walk_to(const Graph* g, int cur, const float x[3], int* steps) {
    for (int it = 0; it < WALK_CAP; ++it) {
        const int e0 = g->off[cur], n = g->off[cur + 1] - e0 + 1;
        float bd = KINF;
        int bk = INT_MAX;
        for (int e = 0; e < n; ++e) {
            const int k = neighbor(g, cur, e0, e);
            float v[3];
            offset_to(g->p, k, x, v);
            const float dk = dot3c(v[0], v[1], v[2], v[0], v[1], v[2]);
            if (dk < bd || (dk == bd && k < bk)) bd = dk, bk = k;
        }
        if (bk == cur) break;
        cur = bk;
        ++*steps;
    }
    return cur;
}

/* Exit face of cell i along the ray (foam.cu:185-209). */
static void exit_face(const Graph* g, int i, const float o[3], const float d[3], float* t_exit, int* next) {
    const int64_t i3 = 3 * (int64_t)i;
    const float pi[3] = {g->p[i3], g->p[i3 + 1], g->p[i3 + 2]};
    const int e0 = g->off[i], e1 = g->off[i + 1];
    float bt = KINF;
    int bk = INT_MAX;
    for (int e = e0; e < e1; ++e) {
        const int j = g->adj[e];
        const int64_t j3 = 3 * (int64_t)j;
        float n[3], m[3];
        for (int a = 0; a < 3; ++a) {
            const float pj = g->p[j3 + a];
            n[a] = pj - pi[a];
            m[a] = fmaf(0.5f, pj + pi[a], -o[a]);
        }
        const float dn = dot3c(n[0], n[1], n[2], d[0], d[1], d[2]);
        if (dn > 0.f) {
            const float t = dot3c(m[0], m[1], m[2], n[0], n[1], n[2]) / dn;
            if (t < bt || (t == bt && j < bk)) bt = t, bk = j;
        }
    }
    *t_exit = bt, *next = bk;
}

/* foam.cu:211-221 */
static float density_at(const Graph* g, const Field* F, int i, const float x[3]) {
    const int e0 = g->off[i], n = g->off[i + 1] - e0 + 1;
    float s = 0.f;
    for (int e = 0; e < n; ++e) {
        const int k = neighbor(g, i, e0, e);
        float v[3];
        offset_to(g->p, k, x, v);
        s += expf(fminf(F->raw[k], 30.f) - 0.5f * maha(F->dA, k, v));
    }
    return s;
}

typedef struct {
    float t, x[3];
    int site;
    float sigma;
    int has_c;
    float C[3], mmin, inv_a;
} Sample;

/* Normalised blend of the neighbourhood colours (foam.cu:224-249). */
static void color_at(const Graph* g, const Field* F, Sample* P, const float b[16]) {
    const int i = P->site;
    const int e0 = g->off[i], n = g->off[i + 1] - e0 + 1;
    const int nb = (F->deg + 1) * (F->deg + 1);
    float ml = KINF;
    for (int e = 0; e < n; ++e) {
        const int k = neighbor(g, i, e0, e);
        float v[3];
        offset_to(g->p, k, P->x, v);
        ml = fminf(ml, maha(F->cA, k, v));
    }
    P->mmin = ml;
    float A = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
    for (int e = 0; e < n; ++e) {
        const int k = neighbor(g, i, e0, e);
        float v[3];
        offset_to(g->p, k, P->x, v);
        const float a = expf(-0.5f * (maha(F->cA, k, v) - P->mmin));
        float c[3];
        sh_eval(F->sh, k, b, nb, c);
        A += a, cr += a * fmaxf(c[0], 0.f), cg += a * fmaxf(c[1], 0.f), cb += a * fmaxf(c[2], 0.f);
    }
    P->inv_a = 1.f / A;
    P->C[0] = cr * P->inv_a, P->C[1] = cg * P->inv_a, P->C[2] = cb * P->inv_a;
    P->has_c = 1;
}

static void make_sample(const Graph* g, const Field* F, const float o[3], const float d[3], float t, int site,
                        Sample* P) {
    P->t = t;
    for (int a = 0; a < 3; ++a) P->x[a] = fmaf(t, d[a], o[a]);
    P->site = site;
    P->sigma = density_at(g, F, site, P->x);
    P->has_c = 0;
    P->C[0] = P->C[1] = P->C[2] = 0.f;
    P->mmin = 0.f, P->inv_a = 0.f;
}

/* foam.cu:262-270 */
static int next_sample(const Graph* g, const Field* F, const float o[3], const float d[3], float far,
                       const Sample* P, int cur, Sample* Q) {
    float t_exit;
    int nxt;
    exit_face(g, cur, o, d, &t_exit, &nxt);
    const int last = nxt == INT_MAX || t_exit >= far;
    make_sample(g, F, o, d, last ? far : fmaxf(t_exit, P->t), last ? cur : nxt, Q);
    return last;
}

/* foam.cu:276-300 */
static void store_sample(float* rec, int64_t r, int K, int s, const Sample* P) {
    if (rec == NULL || s >= K) return;
    float* q = rec + (r * K + s) * RECORD;
    q[0] = P->t;
    int32_t site = P->site;
    memcpy(&q[1], &site, 4);
    q[2] = P->sigma;
    q[3] = P->C[0], q[4] = P->C[1], q[5] = P->C[2];
    q[6] = P->mmin;
    q[7] = P->has_c ? P->inv_a : 0.f;
}

static void load_sample(const float* rec, int64_t r, int K, int s, const float o[3], const float d[3],
                        Sample* P) {
    const float* q = rec + (r * K + s) * RECORD;
    P->t = q[0];
    for (int a = 0; a < 3; ++a) P->x[a] = fmaf(P->t, d[a], o[a]);
    memcpy(&P->site, &q[1], 4);
    P->sigma = q[2];
    P->C[0] = q[3], P->C[1] = q[4], P->C[2] = q[5];
    P->mmin = q[6];
    P->inv_a = q[7];
    P->has_c = P->inv_a > 0.f;
}

static inline void scatter_conic(float* gA, int k, float gm, const float v[3]) {
    float* a = gA + 6 * (int64_t)k;
    a[0] += gm * v[0] * v[0];
    a[1] += 2.f * gm * v[0] * v[1];
    a[2] += 2.f * gm * v[0] * v[2];
    a[3] += gm * v[1] * v[1];
    a[4] += 2.f * gm * v[1] * v[2];
    a[5] += gm * v[2] * v[2];
}

typedef struct {
    float *g_raw, *g_dA, *g_cA, *g_sh;
} Grads;

/* Gradients of one sample: gs = dL/dsigma, gC = dL/dC (foam.cu:303-343). */
static void scatter_sample(const Graph* g, const Field* F, const Sample* P, float gs, const float gC[3],
                           const float b[16], const Grads* G) {
    const int i = P->site;
    const int e0 = g->off[i], n = g->off[i + 1] - e0 + 1;
    if (gs != 0.f) {
        for (int e = 0; e < n; ++e) {
            const int q = neighbor(g, i, e0, e);
            float v[3];
            offset_to(g->p, q, P->x, v);
            const float gc = gs * expf(fminf(F->raw[q], 30.f) - 0.5f * maha(F->dA, q, v));
            if (fabsf(gc) > 1e-12f) {
                lock_site(q);
                G->g_raw[q] += gc;
                scatter_conic(G->g_dA, q, -0.5f * gc, v);
                unlock_site(q);
            }
        }
    }
    if (!P->has_c || (gC[0] == 0.f && gC[1] == 0.f && gC[2] == 0.f)) return;
    const int nb = (F->deg + 1) * (F->deg + 1);
    const float gCC = gC[0] * P->C[0] + gC[1] * P->C[1] + gC[2] * P->C[2];
    for (int e = 0; e < n; ++e) {
        const int q = neighbor(g, i, e0, e);
        float v[3];
        offset_to(g->p, q, P->x, v);
        const float a = expf(-0.5f * (maha(F->cA, q, v) - P->mmin)) * P->inv_a;
        if (a < MIN_WEIGHT) continue;
        float c[3];
        sh_eval(F->sh, q, b, nb, c);
        const float dc0 = c[0] > 0.f ? a * gC[0] : 0.f, dc1 = c[1] > 0.f ? a * gC[1] : 0.f,
                    dc2 = c[2] > 0.f ? a * gC[2] : 0.f;
        const float ga = gC[0] * fmaxf(c[0], 0.f) + gC[1] * fmaxf(c[1], 0.f) + gC[2] * fmaxf(c[2], 0.f);
        const float gm = -0.5f * a * (ga - gCC);
        lock_site(q);
        float* gsh = G->g_sh + 48 * (int64_t)q;
        for (int j = 0; j < nb; ++j) {
            gsh[3 * j] += b[j] * dc0;
            gsh[3 * j + 1] += b[j] * dc1;
            gsh[3 * j + 2] += b[j] * dc2;
        }
        if (gm != 0.f) scatter_conic(G->g_cA, q, gm, v);
        unlock_site(q);
    }
}

/* ------------------------------------------------------------------------------------- foam */

typedef struct {
    Graph g;
    Field F;
    const float *o, *d, *near, *mid, *far;
    const int32_t* start;
    float t_thresh, w_thresh;
    int K;
    float *rgb, *T, *depth, *rec;
    int32_t* stats;
    /* backward */
    const float *rgb_in, *T_in, *g_rgb, *g_T;
    const float* rec_in;
    const int32_t* stats_in;
    Grads G;
    /* march */
    float dt;
    int n_bg;
} Ctx;

static void foam_forward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    const float o[3] = {c->o[3 * r], c->o[3 * r + 1], c->o[3 * r + 2]};
    const float d[3] = {c->d[3 * r], c->d[3 * r + 1], c->d[3 * r + 2]};
    const float near = c->near[r], far = c->far[r];
    float b[16];
    sh_basis(d[0], d[1], d[2], c->F.deg, b);
    int walk_steps = 0, n_samples = 1, n_color = 0;
    float x0[3];
    for (int a = 0; a < 3; ++a) x0[a] = fmaf(near, d[a], o[a]);
    int cur = walk_to(&c->g, c->start[r], x0, &walk_steps);
    Sample P, Q;
    make_sample(&c->g, &c->F, o, d, near, cur, &P);
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f}, dep = 0.f;
    for (int it = 0; it < MAX_CELLS; ++it) {
        const int last = next_sample(&c->g, &c->F, o, d, far, &P, cur, &Q);
        ++n_samples;
        const float delta = Q.t - P.t;
        const float alpha = 1.f - expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        if (w > c->w_thresh) {
            if (!P.has_c) color_at(&c->g, &c->F, &P, b);
            color_at(&c->g, &c->F, &Q, b);
            for (int a = 0; a < 3; ++a) acc[a] += w * 0.5f * (P.C[a] + Q.C[a]);
            dep += w * 0.5f * (P.t + Q.t);
            ++n_color;
        }
        T *= 1.f - alpha;
        store_sample(c->rec, r, c->K, n_samples - 2, &P);
        P = Q;
        cur = Q.site;
        if (last || T < c->t_thresh) break;
    }
    store_sample(c->rec, r, c->K, n_samples - 1, &P);
    for (int a = 0; a < 3; ++a) c->rgb[3 * r + a] = acc[a];
    c->T[r] = T;
    c->depth[r] = dep;
    c->stats[3 * r] = n_samples, c->stats[3 * r + 1] = n_color, c->stats[3 * r + 2] = walk_steps;
}

static void foam_backward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    const float o[3] = {c->o[3 * r], c->o[3 * r + 1], c->o[3 * r + 2]};
    const float d[3] = {c->d[3 * r], c->d[3 * r + 1], c->d[3 * r + 2]};
    const float near = c->near[r], far = c->far[r];
    float b[16];
    sh_basis(d[0], d[1], d[2], c->F.deg, b);
    const float gR[3] = {c->g_rgb[3 * r], c->g_rgb[3 * r + 1], c->g_rgb[3 * r + 2]};
    const float fg[3] = {c->rgb_in[3 * r], c->rgb_in[3 * r + 1], c->rgb_in[3 * r + 2]};
    const float gT_final = c->g_T[r] * c->T_in[r];
    const int K = c->K;
    const int n_stored = c->rec_in != NULL && c->stats_in[3 * r] <= K ? c->stats_in[3 * r] : 0;
    Sample P, Q;
    int cur = 0;
    if (n_stored > 0) {
        load_sample(c->rec_in, r, K, 0, o, d, &P);
    } else {
        int walk_steps = 0;
        float x0[3];
        for (int a = 0; a < 3; ++a) x0[a] = fmaf(near, d[a], o[a]);
        cur = walk_to(&c->g, c->start[r], x0, &walk_steps);
        make_sample(&c->g, &c->F, o, d, near, cur, &P);
    }
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f};
    float gs_pending = 0.f, gC_pending[3] = {0.f, 0.f, 0.f};
    for (int it = 0; it < MAX_CELLS; ++it) {
        int last;
        if (n_stored > 0) {
            if (it + 1 >= n_stored) break;
            load_sample(c->rec_in, r, K, it + 1, o, d, &Q);
            last = it + 2 >= n_stored;
        } else {
            last = next_sample(&c->g, &c->F, o, d, far, &P, cur, &Q);
        }
        const float delta = Q.t - P.t;
        const float alpha = 1.f - expf(-0.5f * (P.sigma + Q.sigma) * delta);
        const float w = T * alpha;
        const float T_next = T * (1.f - alpha);
        const int active = w > c->w_thresh;
        float cc[3] = {0.f, 0.f, 0.f};
        if (active) {
            if (!P.has_c) color_at(&c->g, &c->F, &P, b);
            if (!Q.has_c) color_at(&c->g, &c->F, &Q, b);
            for (int a = 0; a < 3; ++a) {
                cc[a] = 0.5f * (P.C[a] + Q.C[a]);
                acc[a] += w * cc[a];
            }
        }
        float g_sbar = 0.f;
        for (int a = 0; a < 3; ++a) g_sbar += gR[a] * (T_next * cc[a] - (fg[a] - acc[a]));
        g_sbar = delta * (g_sbar - gT_final);
        const float gc_half[3] = {active ? 0.5f * w * gR[0] : 0.f, active ? 0.5f * w * gR[1] : 0.f,
                                  active ? 0.5f * w * gR[2] : 0.f};
        const float gC_P[3] = {gC_pending[0] + gc_half[0], gC_pending[1] + gc_half[1], gC_pending[2] + gc_half[2]};
        scatter_sample(&c->g, &c->F, &P, gs_pending + 0.5f * g_sbar, gC_P, b, &c->G);
        gs_pending = 0.5f * g_sbar;
        for (int a = 0; a < 3; ++a) gC_pending[a] = gc_half[a];
        T = T_next;
        P = Q;
        cur = Q.site;
        if (last || T < c->t_thresh) break;
    }
    scatter_sample(&c->g, &c->F, &P, gs_pending, gC_pending, b, &c->G);
}

static void fill_common(Ctx* c, const float* points, const int32_t* offsets, const int32_t* adj, const float* raw,
                        const float* dA, const float* cA, const float* sh, int sh_deg, const float* o,
                        const float* d, const int32_t* start, const float* near, const float* far, float t_thresh,
                        float w_thresh) {
    memset(c, 0, sizeof(*c));
    c->g.p = points, c->g.off = offsets, c->g.adj = adj;
    c->F.raw = raw, c->F.dA = dA, c->F.cA = cA, c->F.sh = sh, c->F.deg = sh_deg;
    c->o = o, c->d = d, c->start = start, c->near = near, c->far = far;
    c->t_thresh = t_thresh, c->w_thresh = w_thresh;
}

int vgo_foam_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                     const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                     const float* o, const float* d, const int32_t* start, const float* near, const float* far,
                     int64_t n_rays, float t_thresh, float w_thresh, int record_cap, float* rgb, float* T,
                     float* depth, int32_t* stats, float* rec, int n_threads) {
    (void)n_sites;
    if (sh_deg < 0 || sh_deg > 3) return 1;
    Ctx c;
    fill_common(&c, points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh);
    c.K = record_cap > 0 ? record_cap : 0;
    c.rec = record_cap > 0 ? rec : NULL;
    c.rgb = rgb, c.T = T, c.depth = depth, c.stats = stats;
    parallel_for(n_rays, n_threads, &c, foam_forward_ray);
    return 0;
}

int vgo_foam_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                      const float* o, const float* d, const int32_t* start, const float* near, const float* far,
                      int64_t n_rays, float t_thresh, float w_thresh, const float* rgb, const float* T,
                      const float* g_rgb, const float* g_T, const float* rec, int record_cap,
                      const int32_t* stats, float* g_raw, float* g_dA, float* g_cA, float* g_sh,
                      int n_threads) {
    (void)n_sites;
    if (sh_deg < 0 || sh_deg > 3) return 1;
    Ctx c;
    fill_common(&c, points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh);
    c.rgb_in = rgb, c.T_in = T, c.g_rgb = g_rgb, c.g_T = g_T;
    c.K = record_cap > 0 ? record_cap : 0;
    c.rec_in = record_cap > 0 ? rec : NULL;
    c.stats_in = stats;
    c.G.g_raw = g_raw, c.G.g_dA = g_dA, c.G.g_cA = g_cA, c.G.g_sh = g_sh;
    g_use_locks = n_threads > 1;
    parallel_for(n_rays, n_threads, &c, foam_backward_ray);
    g_use_locks = 0;
    return 0;
}

/* ------------------------------------------------------------------------------------ march */

typedef struct {
    float o[3], d[3];
    float near, mid, far;
    int n_in, n_total;
} MRay;

/* march.cu:134-141 */
static void load_mray(const Ctx* c, int64_t r, MRay* R) {
    for (int a = 0; a < 3; ++a) R->o[a] = c->o[3 * r + a], R->d[a] = c->d[3 * r + a];
    R->near = c->near[r], R->mid = c->mid[r], R->far = c->far[r];
    R->n_in = R->mid > R->near ? (int)ceilf((R->mid - R->near) / c->dt) : 0;
    R->n_total = R->n_in + c->n_bg;
}

/* march.cu:143-153 */
static void sample_at(const MRay* R, const Ctx* c, int k, float* t, float* delta) {
    if (k < R->n_in) {
        const float t0 = fmaf((float)k, c->dt, R->near), t1 = fminf(t0 + c->dt, R->mid);
        *t = 0.5f * (t0 + t1), *delta = t1 - t0;
    } else {
        const float i0 = 1.f / R->mid, i1 = 1.f / R->far;
        const float u0 = (float)(k - R->n_in) / c->n_bg, u1 = (float)(k - R->n_in + 1) / c->n_bg;
        *t = 1.f / fmaf(0.5f * (u0 + u1), i1 - i0, i0);
        *delta = 1.f / fmaf(u1, i1 - i0, i0) - 1.f / fmaf(u0, i1 - i0, i0);
    }
}

/* march.cu:195-219 */
static void color_at_x(const Graph* g, const Field* F, int i, const float x[3], const float b[16], float C[3],
                       float* mmin, float* inv_a) {
    Sample P;
    P.site = i;
    memcpy(P.x, x, sizeof(P.x));
    color_at(g, F, &P, b);
    memcpy(C, P.C, sizeof(P.C));
    *mmin = P.mmin, *inv_a = P.inv_a;
}

static void march_forward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    MRay R;
    load_mray(c, r, &R);
    float b[16];
    sh_basis(R.d[0], R.d[1], R.d[2], c->F.deg, b);
    int cur = c->start[r], n_samples = 0, n_color = 0, walk_steps = 0;
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f}, dep = 0.f;
    for (int k = 0; k < R.n_total; ++k) {
        float t, delta, x[3];
        sample_at(&R, c, k, &t, &delta);
        for (int a = 0; a < 3; ++a) x[a] = fmaf(t, R.d[a], R.o[a]);
        cur = walk_to(&c->g, cur, x, &walk_steps);
        const float alpha = 1.f - expf(-density_at(&c->g, &c->F, cur, x) * delta);
        const float w = T * alpha;
        ++n_samples;
        if (w > c->w_thresh) {
            float C[3], mmin, inv_a;
            color_at_x(&c->g, &c->F, cur, x, b, C, &mmin, &inv_a);
            for (int a = 0; a < 3; ++a) acc[a] += w * C[a];
            dep += w * t;
            ++n_color;
        }
        T *= 1.f - alpha;
        if (T < c->t_thresh) break;
    }
    for (int a = 0; a < 3; ++a) c->rgb[3 * r + a] = acc[a];
    c->T[r] = T;
    c->depth[r] = dep;
    c->stats[3 * r] = n_samples, c->stats[3 * r + 1] = n_color, c->stats[3 * r + 2] = walk_steps;
}

static void march_backward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    MRay R;
    load_mray(c, r, &R);
    float b[16];
    sh_basis(R.d[0], R.d[1], R.d[2], c->F.deg, b);
    const float gR[3] = {c->g_rgb[3 * r], c->g_rgb[3 * r + 1], c->g_rgb[3 * r + 2]};
    const float fg[3] = {c->rgb_in[3 * r], c->rgb_in[3 * r + 1], c->rgb_in[3 * r + 2]};
    const float gT_final = c->g_T[r] * c->T_in[r];
    int cur = c->start[r], walk_steps = 0;
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < R.n_total; ++k) {
        float t, delta, x[3];
        sample_at(&R, c, k, &t, &delta);
        for (int a = 0; a < 3; ++a) x[a] = fmaf(t, R.d[a], R.o[a]);
        cur = walk_to(&c->g, cur, x, &walk_steps);
        const float alpha = 1.f - expf(-density_at(&c->g, &c->F, cur, x) * delta);
        const float w = T * alpha;
        const float T_next = T * (1.f - alpha);
        Sample P;
        memset(&P, 0, sizeof(P));
        P.site = cur;
        memcpy(P.x, x, sizeof(P.x));
        const int active = w > c->w_thresh;
        if (active) {
            color_at(&c->g, &c->F, &P, b);
            for (int a = 0; a < 3; ++a) acc[a] += w * P.C[a];
        }
        float gsig = 0.f;
        for (int a = 0; a < 3; ++a) gsig += gR[a] * (T_next * P.C[a] - (fg[a] - acc[a]));
        gsig = delta * (gsig - gT_final);
        const float gC[3] = {active ? w * gR[0] : 0.f, active ? w * gR[1] : 0.f, active ? w * gR[2] : 0.f};
        scatter_sample(&c->g, &c->F, &P, gsig, gC, b, &c->G);
        T = T_next;
        if (T < c->t_thresh) break;
    }
}

int vgo_march_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                      const float* o, const float* d, const int32_t* start, const float* near, const float* mid,
                      const float* far, int64_t n_rays, float dt, int n_bg, float t_thresh, float w_thresh,
                      float* rgb, float* T, float* depth, int32_t* stats, int n_threads) {
    (void)n_sites;
    if (sh_deg < 0 || sh_deg > 3) return 1;
    Ctx c;
    fill_common(&c, points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh);
    c.mid = mid, c.dt = dt, c.n_bg = n_bg;
    c.rgb = rgb, c.T = T, c.depth = depth, c.stats = stats;
    parallel_for(n_rays, n_threads, &c, march_forward_ray);
    return 0;
}

int vgo_march_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                       const float* raw, const float* dA, const float* cA, const float* sh, int sh_deg,
                       const float* o, const float* d, const int32_t* start, const float* near,
                       const float* mid, const float* far, int64_t n_rays, float dt, int n_bg,
                       float t_thresh, float w_thresh, const float* rgb, const float* T, const float* g_rgb,
                       const float* g_T, float* g_raw, float* g_dA, float* g_cA, float* g_sh, int n_threads) {
    (void)n_sites;
    if (sh_deg < 0 || sh_deg > 3) return 1;
    Ctx c;
    fill_common(&c, points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh);
    c.mid = mid, c.dt = dt, c.n_bg = n_bg;
    c.rgb_in = rgb, c.T_in = T, c.g_rgb = g_rgb, c.g_T = g_T;
    c.G.g_raw = g_raw, c.G.g_dA = g_dA, c.G.g_cA = g_cA, c.G.g_sh = g_sh;
    g_use_locks = n_threads > 1;
    parallel_for(n_rays, n_threads, &c, march_backward_ray);
    g_use_locks = 0;
    return 0;
}

/* ------------------------------------------------------------------------------------ conic */

/* vgf.cu:340-344 */
static void quat_to_rot(float w, float a, float b, float c, float R[9]) {
    R[0] = 1.f - 2.f * (b * b + c * c), R[1] = 2.f * (a * b - w * c), R[2] = 2.f * (a * c + w * b);
    R[3] = 2.f * (a * b + w * c), R[4] = 1.f - 2.f * (a * a + c * c), R[5] = 2.f * (b * c - w * a);
    R[6] = 2.f * (a * c - w * b), R[7] = 2.f * (b * c + w * a), R[8] = 1.f - 2.f * (a * a + b * b);
}

typedef struct {
    float qn[4], qnorm, R[9], iv[3], s2[3];
} ConicLocal;

/* vgf.cu:350-362 */
static void conic_local(const float* ls, const float* quat, int64_t i, float floor2, ConicLocal* L) {
    const float* q = quat + 4 * i;
    L->qnorm = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
    for (int k = 0; k < 4; ++k) L->qn[k] = q[k] / L->qnorm;
    quat_to_rot(L->qn[0], L->qn[1], L->qn[2], L->qn[3], L->R);
    for (int k = 0; k < 3; ++k) {
        const float s = expf(2.f * fminf(fmaxf(ls[3 * i + k], -20.f), 20.f));
        L->s2[k] = s;
        L->iv[k] = 1.f / (s + floor2);
    }
}

void vgo_conic_forward(const float* ls, const float* quat, int64_t n, float floor, float* A) {
    static const int ab[6][2] = {{0, 0}, {0, 1}, {0, 2}, {1, 1}, {1, 2}, {2, 2}};
    const float floor2 = floor * floor;
    for (int64_t i = 0; i < n; ++i) {
        ConicLocal L;
        conic_local(ls, quat, i, floor2, &L);
        const float* R = L.R;
        for (int e = 0; e < 6; ++e) {
            const int a = ab[e][0], b = ab[e][1];
            A[6 * i + e] = R[3 * a] * R[3 * b] * L.iv[0] + R[3 * a + 1] * R[3 * b + 1] * L.iv[1] +
                           R[3 * a + 2] * R[3 * b + 2] * L.iv[2];
        }
    }
}

/* vgf.cu:382-421 */
void vgo_conic_backward(const float* ls, const float* quat, int64_t n, float floor, const float* gA, float* g_ls,
                        float* g_quat) {
    const float floor2 = floor * floor;
    for (int64_t i = 0; i < n; ++i) {
        ConicLocal L;
        conic_local(ls, quat, i, floor2, &L);
        const float* R = L.R;
        const float* g = gA + 6 * i;
        const float G[9] = {g[0], 0.5f * g[1], 0.5f * g[2], 0.5f * g[1], g[3], 0.5f * g[4], 0.5f * g[2], 0.5f * g[4], g[5]};
        float GR[9];
        for (int a = 0; a < 3; ++a)
            for (int k = 0; k < 3; ++k) GR[3 * a + k] = G[3 * a] * R[k] + G[3 * a + 1] * R[3 + k] + G[3 * a + 2] * R[6 + k];
        for (int k = 0; k < 3; ++k) {
            const float g_iv = R[k] * GR[k] + R[3 + k] * GR[3 + k] + R[6 + k] * GR[6 + k];
            g_ls[3 * i + k] = g_iv * (-2.f * L.s2[k] * L.iv[k] * L.iv[k]);
        }
        float dR[9];
        for (int a = 0; a < 3; ++a)
            for (int k = 0; k < 3; ++k) dR[3 * a + k] = 2.f * GR[3 * a + k] * L.iv[k];
        const float w = L.qn[0], x = L.qn[1], y = L.qn[2], z = L.qn[3];
        float dq[4];
        dq[0] = 2.f * (-z * dR[1] + y * dR[2] + z * dR[3] - x * dR[5] - y * dR[6] + x * dR[7]);
        dq[1] = 2.f * (y * dR[1] + z * dR[2] + y * dR[3] - 2.f * x * dR[4] - w * dR[5] + z * dR[6] + w * dR[7] -
                       2.f * x * dR[8]);
        dq[2] = 2.f * (-2.f * y * dR[0] + x * dR[1] + w * dR[2] + x * dR[3] + z * dR[5] - w * dR[6] + z * dR[7] -
                       2.f * y * dR[8]);
        dq[3] = 2.f * (-2.f * z * dR[0] - w * dR[1] + x * dR[2] + w * dR[3] - 2.f * z * dR[4] + y * dR[5] +
                       x * dR[6] + y * dR[7]);
        const float proj = dq[0] * w + dq[1] * x + dq[2] * y + dq[3] * z;
        for (int k = 0; k < 4; ++k) g_quat[4 * i + k] = (dq[k] - proj * L.qn[k]) / L.qnorm;
    }
}

/* ------------------------------------------------------------------ NeRF-sampler field kernels */

/* vgf.cu:51-78: greedy walk of every sorted sample of a ray from the previous sample's site; a step
 * moves to the first neighbour (adjacency order) strictly closer than the best so far. */
int vgo_walk(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites, const float* o,
             const float* d, const float* z, const int32_t* start, int64_t n_rays, int n_samples, int32_t* site,
             int32_t* steps) {
    (void)n_sites;
    for (int64_t r = 0; r < n_rays; ++r) {
        const float* orr = o + 3 * r;
        const float* dr = d + 3 * r;
        int cur = start[r], total = 0;
        for (int s = 0; s < n_samples; ++s) {
            const float t = z[r * n_samples + s];
            const float x[3] = {fmaf(t, dr[0], orr[0]), fmaf(t, dr[1], orr[1]), fmaf(t, dr[2], orr[2])};
            const float* pc = points + 3 * (int64_t)cur;
            const float u0 = x[0] - pc[0], u1 = x[1] - pc[1], u2 = x[2] - pc[2];
            float best_d = dot3c(u0, u1, u2, u0, u1, u2);
            for (int it = 0; it < WALK_CAP; ++it) {
                int best = cur;
                for (int e = offsets[cur]; e < offsets[cur + 1]; ++e) {
                    const int q = adj[e];
                    const float* pq = points + 3 * (int64_t)q;
                    const float v0 = x[0] - pq[0], v1 = x[1] - pq[1], v2 = x[2] - pq[2];
                    const float dq = dot3c(v0, v1, v2, v0, v1, v2);
                    if (dq < best_d) best_d = dq, best = q;
                }
                if (best == cur) break;
                cur = best;
                ++total;
            }
            site[r * n_samples + s] = cur;
        }
        steps[r] = total;
    }
    return 0;
}

typedef struct {
    float v[3], y[3], is2[3], qn[4], qnorm, R[9], m;
} GaussLocal;

/* vgf.cu:99-124: the Gaussian of site i at x, rotation rebuilt from the quaternion. */
static void gauss_local(const float* points, const float* ls, const float* quat, int i, const float x[3],
                        float inv_mult2, GaussLocal* L) {
    const int64_t i3 = 3 * (int64_t)i;
    for (int a = 0; a < 3; ++a) L->v[a] = x[a] - points[i3 + a];
    const float* q = quat + 4 * (int64_t)i;
    L->qnorm = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
    for (int k = 0; k < 4; ++k) L->qn[k] = q[k] / L->qnorm;
    quat_to_rot(L->qn[0], L->qn[1], L->qn[2], L->qn[3], L->R);
    L->m = 0.f;
    for (int k = 0; k < 3; ++k) {
        L->y[k] = L->R[k] * L->v[0] + L->R[3 + k] * L->v[1] + L->R[6 + k] * L->v[2];
        const float s = expf(fminf(fmaxf(ls[i3 + k], -20.f), 20.f));
        L->is2[k] = inv_mult2 / (s * s);
        L->m += L->y[k] * L->y[k] * L->is2[k];
    }
}

/* vgf.cu:126-153: dL/dls and dL/dq of one Gaussian from gm = dL/dm (accumulated). */
static void scatter_gauss_grad(const GaussLocal* L, float gm, int i, float* g_ls, float* g_quat) {
    const int64_t i3 = 3 * (int64_t)i;
    float yk[3];
    for (int k = 0; k < 3; ++k) {
        yk[k] = 2.f * gm * L->y[k] * L->is2[k];
        g_ls[i3 + k] += -2.f * gm * L->y[k] * L->y[k] * L->is2[k];
    }
    float GR[9];
    for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) GR[3 * a + b] = L->v[a] * yk[b];
    const float w = L->qn[0], x = L->qn[1], y = L->qn[2], z = L->qn[3];
    float dq[4];
    dq[0] = 2.f * (-z * GR[1] + y * GR[2] + z * GR[3] - x * GR[5] - y * GR[6] + x * GR[7]);
    dq[1] = 2.f * (y * GR[1] + z * GR[2] + y * GR[3] - 2.f * x * GR[4] - w * GR[5] + z * GR[6] + w * GR[7] -
                   2.f * x * GR[8]);
    dq[2] = 2.f * (-2.f * y * GR[0] + x * GR[1] + w * GR[2] + x * GR[3] + z * GR[5] - w * GR[6] + z * GR[7] -
                   2.f * y * GR[8]);
    dq[3] = 2.f * (-2.f * z * GR[0] - w * GR[1] + x * GR[2] + w * GR[3] - 2.f * z * GR[4] + y * GR[5] + x * GR[6] +
                   y * GR[7]);
    const float proj = dq[0] * w + dq[1] * x + dq[2] * y + dq[3] * z;
    for (int k = 0; k < 4; ++k) g_quat[4 * (int64_t)i + k] += (dq[k] - proj * L->qn[k]) / L->qnorm;
}

/* neighbourhood {i} U adj(i) in the reference's order (vgf.cu:155-161) */
static inline int nbhd(const int32_t* offsets, const int32_t* adj, int i, int j) {
    return j == 0 ? i : adj[offsets[i] + j - 1];
}

/* vgf.cu:163-177 */
int vgo_density_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                        const float* raw, const float* ls, const float* quat, const float* x, const int32_t* site,
                        int64_t m, double scale_mult, float* sigma) {
    (void)n_sites;
    const float inv_mult2 = (float)(1.0 / (scale_mult * scale_mult));
    for (int64_t t = 0; t < m; ++t) {
        const int i = site[t];
        const int n = offsets[i + 1] - offsets[i] + 1;
        float s = 0.f;
        for (int j = 0; j < n; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            GaussLocal L;
            gauss_local(points, ls, quat, k, x + 3 * t, inv_mult2, &L);
            s += expf(fminf(raw[k], 30.f) - 0.5f * L.m);
        }
        sigma[t] = s;
    }
    return 0;
}

/* vgf.cu:179-198 (gradients accumulated into zero-filled outputs) */
int vgo_density_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                         const float* raw, const float* ls, const float* quat, const float* x, const int32_t* site,
                         int64_t m, const float* grad_sigma, float* g_raw, float* g_ls, float* g_quat) {
    (void)n_sites;
    for (int64_t t = 0; t < m; ++t) {
        const float gs = grad_sigma[t];
        if (gs == 0.f) continue;
        const int i = site[t];
        const int n = offsets[i + 1] - offsets[i] + 1;
        for (int j = 0; j < n; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            GaussLocal L;
            gauss_local(points, ls, quat, k, x + 3 * t, 1.f, &L);
            const float c = expf(fminf(raw[k], 30.f) - 0.5f * L.m);
            if (c * fabsf(gs) > 1e-12f) {
                g_raw[k] += gs * c;
                scatter_gauss_grad(&L, -0.5f * gs * c, k, g_ls, g_quat);
            }
        }
    }
    return 0;
}

static void unit_dir(const float* dirs, int64_t t, float d[3]) {
    d[0] = dirs[3 * t], d[1] = dirs[3 * t + 1], d[2] = dirs[3 * t + 2];
    const float inv = 1.f / sqrtf(fmaxf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2], 1e-20f));
    d[0] *= inv, d[1] *= inv, d[2] *= inv;
}

/* vgf.cu:248-282 */
int vgo_color_forward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                      const float* ls, const float* quat, const float* sh, int sh_deg, const float* x,
                      const float* dirs, const int32_t* site, int64_t m, float* rgb) {
    (void)n_sites;
    const int nb = (sh_deg + 1) * (sh_deg + 1);
    for (int64_t t = 0; t < m; ++t) {
        float d[3], b[16];
        unit_dir(dirs, t, d);
        sh_basis(d[0], d[1], d[2], sh_deg, b);
        const int i = site[t];
        const int n = offsets[i + 1] - offsets[i] + 1;
        float mmin = KINF, A = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
        for (int j = 0; j < n; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            GaussLocal L;
            gauss_local(points, ls, quat, k, x + 3 * t, 1.f, &L);
            if (L.m < mmin) {
                const float f = mmin == KINF ? 0.f : expf(-0.5f * (mmin - L.m));
                A *= f, cr *= f, cg *= f, cb *= f;
                mmin = L.m;
            }
            const float a = expf(-0.5f * (L.m - mmin));
            float c[3];
            sh_eval(sh, k, b, nb, c);
            A += a;
            cr += a * fmaxf(c[0], 0.f);
            cg += a * fmaxf(c[1], 0.f);
            cb += a * fmaxf(c[2], 0.f);
        }
        rgb[3 * t] = cr / A, rgb[3 * t + 1] = cg / A, rgb[3 * t + 2] = cb / A;
    }
    return 0;
}

/* vgf.cu:284-335 (gradients accumulated into zero-filled outputs) */
int vgo_color_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                       const float* ls, const float* quat, const float* sh, int sh_deg, const float* x,
                       const float* dirs, const int32_t* site, int64_t m, const float* rgb, const float* grad_rgb,
                       float* g_ls, float* g_quat, float* g_sh) {
    (void)n_sites;
    const int nb = (sh_deg + 1) * (sh_deg + 1);
    for (int64_t t = 0; t < m; ++t) {
        const float gr = grad_rgb[3 * t], gg = grad_rgb[3 * t + 1], gb = grad_rgb[3 * t + 2];
        if (gr == 0.f && gg == 0.f && gb == 0.f) continue;
        const int i = site[t];
        const int n = offsets[i + 1] - offsets[i] + 1;
        float mmin = KINF;
        for (int j = 0; j < n; ++j) {
            GaussLocal L;
            gauss_local(points, ls, quat, nbhd(offsets, adj, i, j), x + 3 * t, 1.f, &L);
            mmin = fminf(mmin, L.m);
        }
        float A = 0.f;
        for (int j = 0; j < n; ++j) {
            GaussLocal L;
            gauss_local(points, ls, quat, nbhd(offsets, adj, i, j), x + 3 * t, 1.f, &L);
            A += expf(-0.5f * (L.m - mmin));
        }
        const float inv_a = 1.f / A;
        const float gCC = gr * rgb[3 * t] + gg * rgb[3 * t + 1] + gb * rgb[3 * t + 2];
        float d[3], b[16];
        unit_dir(dirs, t, d);
        sh_basis(d[0], d[1], d[2], sh_deg, b);
        for (int j = 0; j < n; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            GaussLocal L;
            gauss_local(points, ls, quat, k, x + 3 * t, 1.f, &L);
            const float a = expf(-0.5f * (L.m - mmin)) * inv_a;
            if (a < MIN_WEIGHT) continue;
            float c[3];
            sh_eval(sh, k, b, nb, c);
            const float dc[3] = {c[0] > 0.f ? a * gr : 0.f, c[1] > 0.f ? a * gg : 0.f, c[2] > 0.f ? a * gb : 0.f};
            float* gs = g_sh + 48 * (int64_t)k;
            for (int q = 0; q < nb; ++q)
                for (int ch = 0; ch < 3; ++ch) gs[3 * q + ch] += b[q] * dc[ch];
            const float ga = gr * fmaxf(c[0], 0.f) + gg * fmaxf(c[1], 0.f) + gb * fmaxf(c[2], 0.f);
            const float gm = -0.5f * a * (ga - gCC);
            if (gm != 0.f) scatter_gauss_grad(&L, gm, k, g_ls, g_quat);
        }
    }
    return 0;
}

/* -------------------------------------------------------------------------------- foam_infer */

/* IEEE 754 binary16 -> binary32 (exact). */
static float half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else { /* subnormal: m * 2^-24 */
            float f = (float)m * 5.9604644775390625e-8f;
            memcpy(&bits, &f, 4);
            bits |= s;
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Restatement of the inference renderer (foam_infer.cu:121-361) on the packed inference layout: the
 * same samples, skipping rules (density beyond r2, colour below the r2 lam bound), 8-entry direct-mapped
 * colour cache and per-ray counts as the reference's kernel, in plain C. */
enum { EXACT = 0, BAKED = 1, FUSED = 2 }; /* the API's color_mode values */
#define SLOTS 8                           /* colour cache entries per ray (foam_infer.cu:43) */
#define ATTR 20                           /* floats per site in attr */

typedef struct {
    const float* points4; /* (N, 4) */
    const int32_t *offsets, *nbr, *orig;
    const float* edge;    /* (E, 4), w = half2 (r2, lam) bits */
    const float* attr;    /* (N, 20): density conic (6), min(raw, 30), 0, colour conic (6), 0, 0, baked rgb, 0 */
    const void* sh;
    int sh_half, deg;
    float t_thresh, w_thresh, color_cut;
    int mode, stage;
    const float *o, *d, *near, *far;
    const int32_t *start, *cap;
    float *rgb, *T, *depth;
    int32_t* stats;
} ICtx;

/* tie-break order of sites: their ids before any renumbering */
static inline int rank_of(const ICtx* N, int k) { return N->orig != NULL ? N->orig[k] : k; }

/* (r2, lam) of an edge record */
static inline void record_bounds(const float* rec, float* r2, float* lam) {
    uint32_t bits;
    memcpy(&bits, &rec[3], 4);
    *r2 = half_to_float((uint16_t)(bits & 0xffff));
    *lam = half_to_float((uint16_t)(bits >> 16));
}

/* v^T A v of a conic stored (xx, xy, xz, yy, yz, zz) */
static inline float quad6(const float* A, float vx, float vy, float vz) {
    return A[0] * vx * vx + A[3] * vy * vy + A[5] * vz * vz + 2.f * (A[1] * vx * vy + A[2] * vx * vz + A[4] * vy * vz);
}

/* online normalised blend: sums kept relative to the smallest m so far (foam_infer.cu:81-88) */
typedef struct {
    float m_min, wsum, sum[3];
} Mix;

static inline void mix_reset(Mix* M) { M->m_min = KINF, M->wsum = M->sum[0] = M->sum[1] = M->sum[2] = 0.f; }

static inline void mix_add(Mix* M, float m, const float rgb[3]) {
    if (m < M->m_min) {
        const float shrink = expf(-0.5f * (M->m_min - m));
        M->wsum *= shrink;
        for (int ch = 0; ch < 3; ++ch) M->sum[ch] *= shrink;
        M->m_min = m;
    }
    const float a = expf(-0.5f * (m - M->m_min));
    M->wsum += a;
    for (int ch = 0; ch < 3; ++ch) M->sum[ch] += a * rgb[ch];
}

static inline void mix_mean(const Mix* M, float rgb[3]) {
    const float inv = 1.f / M->wsum;
    for (int ch = 0; ch < 3; ++ch) rgb[ch] = M->sum[ch] * inv;
}

/* max(SH_k(d) + 1/2, 0); each channel sums the basis functions in order (foam_infer.cu:121-149) */
static void clamped_colour(const ICtx* N, int k, const float b[16], float rgb[3]) {
    float f[48];
    for (int i = 0; i < 48; ++i)
        f[i] = N->sh_half ? half_to_float(((const uint16_t*)N->sh)[48 * (int64_t)k + i])
                          : ((const float*)N->sh)[48 * (int64_t)k + i];
    rgb[0] = rgb[1] = rgb[2] = 0.5f;
    for (int j = 0; j < 16; ++j)
        for (int ch = 0; ch < 3; ++ch) rgb[ch] += b[j] * f[3 * j + ch];
    for (int ch = 0; ch < 3; ++ch) rgb[ch] = fmaxf(rgb[ch], 0.f);
}

typedef struct {
    float rgb[SLOTS][3];
    int site[SLOTS]; /* -1: empty */
} SlotCache;

/* entry k mod SLOTS; a miss evaluates the SH and counts one evaluation (foam_infer.cu:157-168) */
static void cache_colour(const ICtx* N, SlotCache* C, int k, const float b[16], float rgb[3], int* n_sh) {
    const int s = k & (SLOTS - 1);
    if (C->site[s] != k) {
        clamped_colour(N, k, b, C->rgb[s]);
        C->site[s] = k;
        ++*n_sh;
    }
    for (int ch = 0; ch < 3; ++ch) rgb[ch] = C->rgb[s][ch];
}

static inline float dist2_to(const float x[3], const float* p) {
    const float v0 = x[0] - p[0], v1 = x[1] - p[1], v2 = x[2] - p[2];
    return dot3c(v0, v1, v2, v0, v1, v2);
}

/* greedy walk to the site nearest to x, equal distances to the smaller rank (foam_infer.cu:176-194) */
static int nearest_site(const ICtx* N, int c, const float x[3], int* steps) {
    for (int it = 0; it < WALK_CAP; ++it) {
        float best = dist2_to(x, N->points4 + 4 * (int64_t)c);
        int arg = c;
        for (int e = N->offsets[c] + 1; e < N->offsets[c + 1]; ++e) {
            const int k = N->nbr[e];
            const float dk = dist2_to(x, N->edge + 4 * (int64_t)e);
            if (dk < best || (dk == best && rank_of(N, k) < rank_of(N, arg))) best = dk, arg = k;
        }
        if (arg == c) break;
        c = arg;
        ++*steps;
    }
    return c;
}

typedef struct {
    float sigma, m_min, t_exit;
    int next;
    Mix mix;
} CellScan;

/* crossing of the face between site pc and neighbour record p along the ray, when d . (p - pc) > 0 */
static int face_crossing(const float* p, const float* pc, const float o[3], const float d[3], float* t) {
    const float n0 = p[0] - pc[0], n1 = p[1] - pc[1], n2 = p[2] - pc[2];
    const float towards = dot3c(n0, n1, n2, d[0], d[1], d[2]);
    if (!(towards > 0.f)) return 0;
    const float h0 = fmaf(0.5f, p[0] + pc[0], -o[0]), h1 = fmaf(0.5f, p[1] + pc[1], -o[1]),
                h2 = fmaf(0.5f, p[2] + pc[2], -o[2]);
    *t = dot3c(h0, h1, h2, n0, n1, n2) / towards;
    return 1;
}

/* one scan of cell c for the sample at o + t d (foam_infer.cu:199-257) */
static void scan_cell(const ICtx* N, int c, float t, const float o[3], const float d[3], const float b[16],
                      SlotCache* cache, int find_exit, CellScan* S, int* n_dens, int* n_sh) {
    const int mixing = N->mode != EXACT;
    const float* pc = N->points4 + 4 * (int64_t)c;
    const float x[3] = {fmaf(t, d[0], o[0]), fmaf(t, d[1], o[1]), fmaf(t, d[2], o[2])};
    S->sigma = 0.f, S->m_min = KINF, S->t_exit = KINF, S->next = INT_MAX;
    mix_reset(&S->mix);
    const int e0 = N->offsets[c];
    for (int e = e0; e < N->offsets[c + 1]; ++e) {
        const float* rec = N->edge + 4 * (int64_t)e;
        const int k = N->nbr[e];
        float tc;
        if (find_exit && e != e0 && face_crossing(rec, pc, o, d, &tc) &&
            (tc < S->t_exit || (tc == S->t_exit && (S->next == INT_MAX || rank_of(N, k) < rank_of(N, S->next)))))
            S->t_exit = tc, S->next = k;
        if (N->stage < 1) continue;
        const float v0 = x[0] - rec[0], v1 = x[1] - rec[1], v2 = x[2] - rec[2];
        const float r2 = dot3c(v0, v1, v2, v0, v1, v2);
        float r2_cut, lam;
        record_bounds(rec, &r2_cut, &lam);
        const float* row = N->attr + ATTR * (int64_t)k;
        if (r2 <= r2_cut) {
            S->sigma += expf(row[6] - 0.5f * quad6(row, v0, v1, v2));
            ++*n_dens;
        }
        if (N->stage < 2) continue;
        const float floor_m = r2 * lam;
        if (mixing ? !(floor_m <= S->mix.m_min + N->color_cut) : !(floor_m < S->m_min)) continue;
        const float m = quad6(row + 8, v0, v1, v2);
        if (!mixing) {
            S->m_min = fminf(S->m_min, m);
            continue;
        }
        if (!(m <= S->mix.m_min + N->color_cut)) continue;
        float rgb[3];
        if (N->mode == BAKED)
            rgb[0] = row[16], rgb[1] = row[17], rgb[2] = row[18];
        else
            cache_colour(N, cache, k, b, rgb, n_sh);
        mix_add(&S->mix, m, rgb);
    }
}

typedef struct {
    float t, sigma, m_min, rgb[3];
    int coloured, cell;
} Point;

/* exact-mode colour of a sample: blend of the neighbours within m_min + color_cut (foam_infer.cu:260-284) */
static void exact_colour(const ICtx* N, Point* s, const float o[3], const float d[3], const float b[16],
                         SlotCache* cache, int* n_sh) {
    const float x[3] = {fmaf(s->t, d[0], o[0]), fmaf(s->t, d[1], o[1]), fmaf(s->t, d[2], o[2])};
    const float limit = s->m_min + N->color_cut;
    float wsum = 0.f, sum[3] = {0.f, 0.f, 0.f};
    for (int e = N->offsets[s->cell]; e < N->offsets[s->cell + 1]; ++e) {
        const float* rec = N->edge + 4 * (int64_t)e;
        const float v0 = x[0] - rec[0], v1 = x[1] - rec[1], v2 = x[2] - rec[2];
        float r2_cut, lam;
        record_bounds(rec, &r2_cut, &lam);
        if (dot3c(v0, v1, v2, v0, v1, v2) * lam > limit) continue;
        const int k = N->nbr[e];
        const float m = quad6(N->attr + ATTR * (int64_t)k + 8, v0, v1, v2);
        if (m > limit) continue;
        const float a = expf(-0.5f * (m - s->m_min));
        float rgb[3];
        cache_colour(N, cache, k, b, rgb, n_sh);
        wsum += a;
        for (int ch = 0; ch < 3; ++ch) sum[ch] += a * rgb[ch];
    }
    const float inv = 1.f / wsum;
    for (int ch = 0; ch < 3; ++ch) s->rgb[ch] = sum[ch] * inv;
    s->coloured = 1;
}

static void take_point(const ICtx* N, Point* s, const CellScan* S, float t, int cell) {
    s->t = t, s->sigma = S->sigma, s->m_min = S->m_min, s->cell = cell;
    s->coloured = N->stage >= 2 && N->mode != EXACT;
    if (s->coloured)
        mix_mean(&S->mix, s->rgb);
    else
        s->rgb[0] = s->rgb[1] = s->rgb[2] = 0.f;
}

/* one ray (foam_infer.cu:286-361) */
static void infer_ray(void* vc, int64_t r) {
    const ICtx* N = (const ICtx*)vc;
    SlotCache cache;
    for (int s = 0; s < SLOTS; ++s) cache.site[s] = -1, cache.rgb[s][0] = cache.rgb[s][1] = cache.rgb[s][2] = 0.f;
    const float o[3] = {N->o[3 * r], N->o[3 * r + 1], N->o[3 * r + 2]};
    const float d[3] = {N->d[3 * r], N->d[3 * r + 1], N->d[3 * r + 2]};
    const float t_near = N->near[r], t_far = N->far[r];
    const int max_samples = N->cap != NULL ? N->cap[r] : INT_MAX;
    float b[16] = {0};
    if (N->stage >= 2 && N->mode != BAKED) sh_basis(d[0], d[1], d[2], N->deg, b);
    int walk_steps = 0, n_dens = 0, n_sh = 0, n_samples = 1, n_coloured = 0;
    const float x_near[3] = {fmaf(t_near, d[0], o[0]), fmaf(t_near, d[1], o[1]), fmaf(t_near, d[2], o[2])};
    const int first = nearest_site(N, N->start[r], x_near, &walk_steps);
    CellScan S;
    scan_cell(N, first, t_near, o, d, b, &cache, 1, &S, &n_dens, &n_sh);
    Point P, Q;
    take_point(N, &P, &S, t_near, first);
    float T = 1.f, fg[3] = {0.f, 0.f, 0.f}, depth = 0.f;
    for (int cell = 0; cell < MAX_CELLS; ++cell) {
        const int last = S.next == INT_MAX || S.t_exit >= t_far || n_samples + 1 >= max_samples;
        const float tQ = last ? t_far : fmaxf(S.t_exit, P.t);
        const int cQ = last ? P.cell : S.next;
        scan_cell(N, cQ, tQ, o, d, b, &cache, !last, &S, &n_dens, &n_sh);
        ++n_samples;
        take_point(N, &Q, &S, tQ, cQ);
        const float alpha = 1.f - expf(-0.5f * (P.sigma + Q.sigma) * (Q.t - P.t));
        const float w = T * alpha;
        if (N->stage >= 2 && w > N->w_thresh) {
            if (N->mode == EXACT) {
                if (!P.coloured) exact_colour(N, &P, o, d, b, &cache, &n_sh);
                exact_colour(N, &Q, o, d, b, &cache, &n_sh);
            }
            for (int a = 0; a < 3; ++a) fg[a] += w * 0.5f * (P.rgb[a] + Q.rgb[a]);
            depth += w * 0.5f * (P.t + Q.t);
            ++n_coloured;
        }
        T *= 1.f - alpha;
        P = Q;
        if (last || T < N->t_thresh) break;
    }
    for (int a = 0; a < 3; ++a) N->rgb[3 * r + a] = fg[a];
    N->T[r] = T;
    N->depth[r] = depth;
    int32_t* out = N->stats + 5 * r;
    out[0] = n_samples, out[1] = n_coloured, out[2] = walk_steps, out[3] = n_dens, out[4] = n_sh;
}

int vgo_foam_infer(const float* points4, const int32_t* offsets, const int32_t* nbr, const float* edge,
                   const float* attr, const void* sh, int sh_half, int sh_deg, int64_t n_sites, const float* o,
                   const float* d, const int32_t* start, const float* near, const float* far, int64_t n_rays,
                   float t_thresh, float w_thresh, float color_cut, int color_mode, int stage, const int32_t* cap,
                   const int32_t* orig, float* rgb, float* T, float* depth, int32_t* stats, int n_threads) {
    (void)n_sites;
    if (color_mode < EXACT || color_mode > FUSED || stage < 0 || stage > 2) return 1;
    ICtx N;
    memset(&N, 0, sizeof(N));
    N.points4 = points4, N.offsets = offsets, N.nbr = nbr, N.edge = edge, N.attr = attr, N.sh = sh;
    N.sh_half = sh_half, N.deg = sh_deg, N.orig = orig, N.cap = cap;
    N.t_thresh = t_thresh, N.w_thresh = w_thresh, N.color_cut = color_cut, N.mode = color_mode, N.stage = stage;
    N.o = o, N.d = d, N.near = near, N.far = far, N.start = start;
    N.rgb = rgb, N.T = T, N.depth = depth, N.stats = stats;
    parallel_for(n_rays, n_threads, &N, infer_ray);
    return 0;
}
