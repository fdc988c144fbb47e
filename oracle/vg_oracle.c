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
    const float* p;        /* (N, 3) site positions */
    const int32_t* off;    /* (N + 1) CSR offsets into adj */
    const int32_t* adj;    /* Delaunay neighbours */
} Graph;

typedef struct {
    const float *raw, *dA, *cA, *sh; /* (N), (N, 6), (N, 6), (N, 16, 3) */
    int deg;
} Field;

/* Real SH basis up to degree 3 with the reference's constants and signs (foam.cu:118-141): per band, a
 * normalisation constant times the Cartesian polynomial of the standard real basis. */
static const float SH_K0 = 0.28209479177387814f, SH_K1 = 0.4886025119029199f, SH_K2XY = 1.0925484305920792f,
                   SH_K2Z = 0.31539156525252005f, SH_K2D = 0.5462742152960396f, SH_K3A = 0.5900435899266435f,
                   SH_K3B = 2.890611442640554f, SH_K3C = 0.4570457994644658f, SH_K3Z = 0.3731763325901154f,
                   SH_K3D = 1.445305721320277f;

static void sh_basis(float x, float y, float z, int deg, float b[16]) {
    memset(b, 0, 16 * sizeof(float));
    b[0] = SH_K0;
    if (deg >= 1) b[1] = -SH_K1 * y, b[2] = SH_K1 * z, b[3] = -SH_K1 * x;
    if (deg < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    b[4] = SH_K2XY * x * y, b[5] = -SH_K2XY * y * z, b[6] = SH_K2Z * (2.f * zz - xx - yy);
    b[7] = -SH_K2XY * x * z, b[8] = SH_K2D * (xx - yy);
    if (deg < 3) return;
    const float ring = 4.f * zz - xx - yy;
    b[9] = -SH_K3A * y * (3.f * xx - yy), b[10] = SH_K3B * x * y * z, b[11] = -SH_K3C * y * ring;
    b[12] = SH_K3Z * z * (2.f * zz - 3.f * xx - 3.f * yy), b[13] = -SH_K3C * x * ring;
    b[14] = SH_K3D * z * (xx - yy), b[15] = -SH_K3A * x * (xx - 3.f * yy);
}

/* SH_k(d) + 1/2 per channel, unclamped, over the first nb basis functions (foam.cu:143-153) */
static inline void sh_eval(const float* sh, int k, const float b[16], int nb, float c[3]) {
    const float* coef = sh + 48 * (int64_t)k;
    for (int ch = 0; ch < 3; ++ch) {
        float sum = 0.5f;
        for (int j = 0; j < nb; ++j) sum += b[j] * coef[3 * j + ch];
        c[ch] = sum;
    }
}

/* v^T A v for the conic of site k stored (xx, xy, xz, yy, yz, zz) (foam.cu:101-105) */
static inline float maha(const float* A, int k, const float v[3]) {
    const float* a = A + 6 * (int64_t)k;
    const float diag = a[0] * v[0] * v[0] + a[3] * v[1] * v[1] + a[5] * v[2] * v[2];
    const float cross = a[1] * v[0] * v[1] + a[2] * v[0] * v[2] + a[4] * v[1] * v[2];
    return diag + 2.f * cross;
}

/* x - p_k */
static inline void offset_to(const float* p, int k, const float x[3], float v[3]) {
    for (int a = 0; a < 3; ++a) v[a] = x[a] - p[3 * (int64_t)k + a];
}

/* member e of the neighbourhood {i} U adj(i): the site itself first, then its neighbours in order */
static inline int member(const Graph* g, int i, int e) { return e == 0 ? i : g->adj[g->off[i] + e - 1]; }
static inline int members(const Graph* g, int i) { return g->off[i + 1] - g->off[i] + 1; }

static inline float dot3(const float a[3], const float b[3]) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }
static inline float dot3_pos(const float g[3], const float c[3]) {
    return g[0] * fmaxf(c[0], 0.f) + g[1] * fmaxf(c[1], 0.f) + g[2] * fmaxf(c[2], 0.f);
}

/* Greedy walk to the site nearest to x: each step goes to the member of the neighbourhood with the
 * smallest (squared distance, index) (foam.cu:163-181). */
static int nearest_walk(const Graph* g, int cur, const float x[3], int* steps) {
    for (int it = 0; it < WALK_CAP; ++it) {
        float best = KINF;
        int arg = INT_MAX;
        for (int e = 0; e < members(g, cur); ++e) {
            const int k = member(g, cur, e);
            float v[3];
            offset_to(g->p, k, x, v);
            const float dk = dot3c(v[0], v[1], v[2], v[0], v[1], v[2]);
            if (dk < best || (dk == best && k < arg)) best = dk, arg = k;
        }
        if (arg == cur) break;
        cur = arg;
        ++*steps;
    }
    return cur;
}

/* The face through which the ray leaves cell i: the smallest (crossing t, index) among the neighbours the
 * ray moves towards, crossing the bisector plane of (p_i, p_j) (foam.cu:185-209). */
static void leave_cell(const Graph* g, int i, const float o[3], const float d[3], float* t_exit, int* next) {
    const float* pi = g->p + 3 * (int64_t)i;
    float best_t = KINF;
    int best_j = INT_MAX;
    for (int e = g->off[i]; e < g->off[i + 1]; ++e) {
        const int j = g->adj[e];
        const float* pj = g->p + 3 * (int64_t)j;
        float nrm[3], half[3];
        for (int a = 0; a < 3; ++a) nrm[a] = pj[a] - pi[a], half[a] = fmaf(0.5f, pj[a] + pi[a], -o[a]);
        const float towards = dot3c(nrm[0], nrm[1], nrm[2], d[0], d[1], d[2]);
        if (!(towards > 0.f)) continue;
        const float t = dot3c(half[0], half[1], half[2], nrm[0], nrm[1], nrm[2]) / towards;
        if (t < best_t || (t == best_t && j < best_j)) best_t = t, best_j = j;
    }
    *t_exit = best_t, *next = best_j;
}

/* sigma(x) = sum over the neighbourhood of exp(min(raw_k, 30) - v^T dA_k v / 2) (foam.cu:211-221) */
static float cell_density(const Graph* g, const Field* F, int i, const float x[3]) {
    float sigma = 0.f;
    for (int e = 0; e < members(g, i); ++e) {
        const int k = member(g, i, e);
        float v[3];
        offset_to(g->p, k, x, v);
        sigma += expf(fminf(F->raw[k], 30.f) - 0.5f * maha(F->dA, k, v));
    }
    return sigma;
}

/* A point of a ray and what is known about it. */
typedef struct {
    float t, x[3];
    int site;
    float sigma;
    int has_c;          /* colour evaluated */
    float C[3];         /* blended colour */
    float mmin, inv_a;  /* smallest colour distance, 1 / sum of colour weights */
} Stop;

/* Colour of the stop: neighbourhood colours max(SH + 1/2, 0) weighted by exp(-(m_k - m_min) / 2),
 * normalised (foam.cu:224-249). */
static void blend_colour(const Graph* g, const Field* F, Stop* P, const float b[16]) {
    const int i = P->site, n = members(g, i), nb = (F->deg + 1) * (F->deg + 1);
    float m_low = KINF;
    for (int e = 0; e < n; ++e) {
        float v[3];
        offset_to(g->p, member(g, i, e), P->x, v);
        m_low = fminf(m_low, maha(F->cA, member(g, i, e), v));
    }
    P->mmin = m_low;
    float wsum = 0.f, sum[3] = {0.f, 0.f, 0.f};
    for (int e = 0; e < n; ++e) {
        const int k = member(g, i, e);
        float v[3], c[3];
        offset_to(g->p, k, P->x, v);
        const float a = expf(-0.5f * (maha(F->cA, k, v) - P->mmin));
        sh_eval(F->sh, k, b, nb, c);
        wsum += a;
        for (int ch = 0; ch < 3; ++ch) sum[ch] += a * fmaxf(c[ch], 0.f);
    }
    P->inv_a = 1.f / wsum;
    for (int ch = 0; ch < 3; ++ch) P->C[ch] = sum[ch] * P->inv_a;
    P->has_c = 1;
}

static void stop_at(const Graph* g, const Field* F, const float o[3], const float d[3], float t, int site, Stop* P) {
    memset(P, 0, sizeof(*P));
    P->t = t;
    for (int a = 0; a < 3; ++a) P->x[a] = fmaf(t, d[a], o[a]);
    P->site = site;
    P->sigma = cell_density(g, F, site, P->x);
}

/* The stop after P in cell cur: its exit face (t clamped to stay monotone), or x(far) when the cell is
 * unbounded ahead or the face lies beyond far; returns whether it is the last (foam.cu:262-270). */
static int advance(const Graph* g, const Field* F, const float o[3], const float d[3], float far, const Stop* P,
                   int cur, Stop* Q) {
    float t_exit;
    int next;
    leave_cell(g, cur, o, d, &t_exit, &next);
    const int last = next == INT_MAX || t_exit >= far;
    if (last)
        stop_at(g, F, o, d, far, cur, Q);
    else
        stop_at(g, F, o, d, fmaxf(t_exit, P->t), next, Q);
    return last;
}

/* record layout (t, site bits, sigma, C rgb, m_min, 1 / sum of weights or 0) (foam.cu:276-300) */
static void write_record(float* rec, int64_t r, int K, int s, const Stop* P) {
    if (rec == NULL || s >= K) return;
    float* q = rec + (r * K + s) * RECORD;
    const int32_t site = P->site;
    q[0] = P->t;
    memcpy(&q[1], &site, 4);
    q[2] = P->sigma;
    for (int ch = 0; ch < 3; ++ch) q[3 + ch] = P->C[ch];
    q[6] = P->mmin;
    q[7] = P->has_c ? P->inv_a : 0.f;
}

static void read_record(const float* rec, int64_t r, int K, int s, const float o[3], const float d[3], Stop* P) {
    const float* q = rec + (r * K + s) * RECORD;
    P->t = q[0];
    for (int a = 0; a < 3; ++a) P->x[a] = fmaf(P->t, d[a], o[a]);
    memcpy(&P->site, &q[1], 4);
    P->sigma = q[2];
    for (int ch = 0; ch < 3; ++ch) P->C[ch] = q[3 + ch];
    P->mmin = q[6];
    P->inv_a = q[7];
    P->has_c = P->inv_a > 0.f;
}

/* dL/dA of a conic term gm v^T A v in storage order (off-diagonal entries count twice) */
static inline void add_conic_grad(float* gA, int k, float gm, const float v[3]) {
    static const int row[6] = {0, 0, 0, 1, 1, 2}, col[6] = {0, 1, 2, 1, 2, 2};
    float* a = gA + 6 * (int64_t)k;
    for (int e = 0; e < 6; ++e) a[e] += (row[e] == col[e] ? gm : 2.f * gm) * v[row[e]] * v[col[e]];
}

typedef struct {
    float *g_raw, *g_dA, *g_cA, *g_sh;
} Grads;

/* Gradients of one stop, gs = dL/dsigma and gC = dL/dC, into the neighbourhood's parameters
 * (foam.cu:303-343). */
static void stop_grads(const Graph* g, const Field* F, const Stop* P, float gs, const float gC[3], const float b[16],
                       const Grads* G) {
    const int i = P->site, n = members(g, i);
    for (int e = 0; gs != 0.f && e < n; ++e) {
        const int k = member(g, i, e);
        float v[3];
        offset_to(g->p, k, P->x, v);
        const float gc = gs * expf(fminf(F->raw[k], 30.f) - 0.5f * maha(F->dA, k, v));
        if (!(fabsf(gc) > 1e-12f)) continue;
        lock_site(k);
        G->g_raw[k] += gc;
        add_conic_grad(G->g_dA, k, -0.5f * gc, v);
        unlock_site(k);
    }
    if (!P->has_c || (gC[0] == 0.f && gC[1] == 0.f && gC[2] == 0.f)) return;
    const int nb = (F->deg + 1) * (F->deg + 1);
    const float gCC = dot3(gC, P->C);
    for (int e = 0; e < n; ++e) {
        const int k = member(g, i, e);
        float v[3], c[3], dc[3];
        offset_to(g->p, k, P->x, v);
        const float a = expf(-0.5f * (maha(F->cA, k, v) - P->mmin)) * P->inv_a;
        if (a < MIN_WEIGHT) continue;
        sh_eval(F->sh, k, b, nb, c);
        for (int ch = 0; ch < 3; ++ch) dc[ch] = c[ch] > 0.f ? a * gC[ch] : 0.f;
        const float gm = -0.5f * a * (dot3_pos(gC, c) - gCC);
        lock_site(k);
        float* gsh = G->g_sh + 48 * (int64_t)k;
        for (int j = 0; j < nb; ++j)
            for (int ch = 0; ch < 3; ++ch) gsh[3 * j + ch] += b[j] * dc[ch];
        if (gm != 0.f) add_conic_grad(G->g_cA, k, gm, v);
        unlock_site(k);
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

static void ray_of(const Ctx* c, int64_t r, float o[3], float d[3]) {
    for (int a = 0; a < 3; ++a) o[a] = c->o[3 * r + a], d[a] = c->d[3 * r + a];
}

/* Trapezoid compositing over the stops of one ray, records of the first K stops (foam.cu:345-393). */
static void foam_forward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    float o[3], d[3], b[16], x_near[3];
    ray_of(c, r, o, d);
    const float near = c->near[r], far = c->far[r];
    sh_basis(d[0], d[1], d[2], c->F.deg, b);
    int walk_steps = 0, n_stops = 1, n_coloured = 0;
    for (int a = 0; a < 3; ++a) x_near[a] = fmaf(near, d[a], o[a]);
    int cur = nearest_walk(&c->g, c->start[r], x_near, &walk_steps);
    Stop P, Q;
    stop_at(&c->g, &c->F, o, d, near, cur, &P);
    float T = 1.f, fg[3] = {0.f, 0.f, 0.f}, depth = 0.f;
    for (int it = 0; it < MAX_CELLS; ++it) {
        const int last = advance(&c->g, &c->F, o, d, far, &P, cur, &Q);
        ++n_stops;
        const float alpha = 1.f - expf(-0.5f * (P.sigma + Q.sigma) * (Q.t - P.t));
        const float w = T * alpha;
        if (w > c->w_thresh) {
            if (!P.has_c) blend_colour(&c->g, &c->F, &P, b);
            blend_colour(&c->g, &c->F, &Q, b);
            for (int ch = 0; ch < 3; ++ch) fg[ch] += w * 0.5f * (P.C[ch] + Q.C[ch]);
            depth += w * 0.5f * (P.t + Q.t);
            ++n_coloured;
        }
        T *= 1.f - alpha;
        write_record(c->rec, r, c->K, n_stops - 2, &P);
        P = Q;
        cur = Q.site;
        if (last || T < c->t_thresh) break;
    }
    write_record(c->rec, r, c->K, n_stops - 1, &P);
    for (int ch = 0; ch < 3; ++ch) c->rgb[3 * r + ch] = fg[ch];
    c->T[r] = T;
    c->depth[r] = depth;
    int32_t* st = c->stats + 3 * r;
    st[0] = n_stops, st[1] = n_coloured, st[2] = walk_steps;
}

/* Front-to-back replay of one ray from its records (or by tracing it again when it has more stops than
 * records): the gradient of the segment opacity is dL/d(sigma bar) = dt (sum_c gR_c (T_{s+1} C_s,c -
 * (fg_c - acc_c)) - g_T T_final), half of it to each end stop; each end stop's colour gets w gR / 2
 * (foam.cu:395-469). */
static void foam_backward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    float o[3], d[3], b[16];
    ray_of(c, r, o, d);
    const float near = c->near[r], far = c->far[r];
    sh_basis(d[0], d[1], d[2], c->F.deg, b);
    const float* gR = c->g_rgb + 3 * r;
    const float* fg = c->rgb_in + 3 * r;
    const float tail = c->g_T[r] * c->T_in[r];
    const int K = c->K;
    const int recorded = c->rec_in != NULL && c->stats_in[3 * r] <= K ? c->stats_in[3 * r] : 0;
    Stop P, Q;
    int cur = 0;
    if (recorded > 0) {
        read_record(c->rec_in, r, K, 0, o, d, &P);
    } else {
        int walk_steps = 0;
        float x_near[3];
        for (int a = 0; a < 3; ++a) x_near[a] = fmaf(near, d[a], o[a]);
        cur = nearest_walk(&c->g, c->start[r], x_near, &walk_steps);
        stop_at(&c->g, &c->F, o, d, near, cur, &P);
    }
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f};
    float carry_sigma = 0.f, carry_colour[3] = {0.f, 0.f, 0.f}; /* P's share from the segment before it */
    for (int it = 0; it < MAX_CELLS; ++it) {
        int last;
        if (recorded > 0) {
            if (it + 1 >= recorded) break;
            read_record(c->rec_in, r, K, it + 1, o, d, &Q);
            last = it + 2 >= recorded;
        } else {
            last = advance(&c->g, &c->F, o, d, far, &P, cur, &Q);
        }
        const float span = Q.t - P.t;
        const float alpha = 1.f - expf(-0.5f * (P.sigma + Q.sigma) * span);
        const float w = T * alpha;
        const float T_after = T * (1.f - alpha);
        const int lit = w > c->w_thresh;
        float mean[3] = {0.f, 0.f, 0.f};
        if (lit) {
            if (!P.has_c) blend_colour(&c->g, &c->F, &P, b);
            if (!Q.has_c) blend_colour(&c->g, &c->F, &Q, b);
            for (int ch = 0; ch < 3; ++ch) {
                mean[ch] = 0.5f * (P.C[ch] + Q.C[ch]);
                acc[ch] += w * mean[ch];
            }
        }
        float g_opacity = 0.f;
        for (int ch = 0; ch < 3; ++ch) g_opacity += gR[ch] * (T_after * mean[ch] - (fg[ch] - acc[ch]));
        g_opacity = span * (g_opacity - tail);
        float share[3], to_P[3];
        for (int ch = 0; ch < 3; ++ch) {
            share[ch] = lit ? 0.5f * w * gR[ch] : 0.f;
            to_P[ch] = carry_colour[ch] + share[ch];
        }
        stop_grads(&c->g, &c->F, &P, carry_sigma + 0.5f * g_opacity, to_P, b, &c->G);
        carry_sigma = 0.5f * g_opacity;
        for (int ch = 0; ch < 3; ++ch) carry_colour[ch] = share[ch];
        T = T_after;
        P = Q;
        cur = Q.site;
        if (last || T < c->t_thresh) break;
    }
    stop_grads(&c->g, &c->F, &P, carry_sigma, carry_colour, b, &c->G);
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

/* The fixed-step schedule of one ray: n_in midpoints of dt steps from near to mid, then n_bg steps evenly
 * spaced in 1/t from mid to far (march.cu:134-153). */
typedef struct {
    float o[3], d[3];
    float near, mid, far;
    int n_in, n_total;
} Schedule;

static void schedule_of(const Ctx* c, int64_t r, Schedule* R) {
    ray_of(c, r, R->o, R->d);
    R->near = c->near[r], R->mid = c->mid[r], R->far = c->far[r];
    R->n_in = R->mid > R->near ? (int)ceilf((R->mid - R->near) / c->dt) : 0;
    R->n_total = R->n_in + c->n_bg;
}

static void schedule_step(const Schedule* R, const Ctx* c, int k, float* t, float* delta) {
    if (k < R->n_in) {
        const float lo = fmaf((float)k, c->dt, R->near), hi = fminf(lo + c->dt, R->mid);
        *t = 0.5f * (lo + hi), *delta = hi - lo;
        return;
    }
    const float inv_mid = 1.f / R->mid, inv_far = 1.f / R->far, span = inv_far - inv_mid;
    const float u_lo = (float)(k - R->n_in) / c->n_bg, u_hi = (float)(k - R->n_in + 1) / c->n_bg;
    *t = 1.f / fmaf(0.5f * (u_lo + u_hi), span, inv_mid);
    *delta = 1.f / fmaf(u_hi, span, inv_mid) - 1.f / fmaf(u_lo, span, inv_mid);
}

/* alpha = 1 - exp(-sigma dt) per step, the colour where w > w_thresh (march.cu:221-262) */
static void march_forward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    Schedule R;
    schedule_of(c, r, &R);
    float b[16];
    sh_basis(R.d[0], R.d[1], R.d[2], c->F.deg, b);
    int cur = c->start[r], n_steps = 0, n_coloured = 0, walk_steps = 0;
    float T = 1.f, fg[3] = {0.f, 0.f, 0.f}, depth = 0.f;
    for (int k = 0; k < R.n_total; ++k) {
        Stop P;
        float t, delta;
        schedule_step(&R, c, k, &t, &delta);
        memset(&P, 0, sizeof(P));
        for (int a = 0; a < 3; ++a) P.x[a] = fmaf(t, R.d[a], R.o[a]);
        P.site = cur = nearest_walk(&c->g, cur, P.x, &walk_steps);
        const float alpha = 1.f - expf(-cell_density(&c->g, &c->F, cur, P.x) * delta);
        const float w = T * alpha;
        ++n_steps;
        if (w > c->w_thresh) {
            blend_colour(&c->g, &c->F, &P, b);
            for (int ch = 0; ch < 3; ++ch) fg[ch] += w * P.C[ch];
            depth += w * t;
            ++n_coloured;
        }
        T *= 1.f - alpha;
        if (T < c->t_thresh) break;
    }
    for (int ch = 0; ch < 3; ++ch) c->rgb[3 * r + ch] = fg[ch];
    c->T[r] = T;
    c->depth[r] = depth;
    int32_t* st = c->stats + 3 * r;
    st[0] = n_steps, st[1] = n_coloured, st[2] = walk_steps;
}

/* the same march again, each step's gradients scattered as it is passed (march.cu:264-345) */
static void march_backward_ray(void* vc, int64_t r) {
    const Ctx* c = (const Ctx*)vc;
    Schedule R;
    schedule_of(c, r, &R);
    float b[16];
    sh_basis(R.d[0], R.d[1], R.d[2], c->F.deg, b);
    const float* gR = c->g_rgb + 3 * r;
    const float* fg = c->rgb_in + 3 * r;
    const float tail = c->g_T[r] * c->T_in[r];
    int cur = c->start[r], walk_steps = 0;
    float T = 1.f, acc[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < R.n_total; ++k) {
        Stop P;
        float t, delta;
        schedule_step(&R, c, k, &t, &delta);
        memset(&P, 0, sizeof(P));
        for (int a = 0; a < 3; ++a) P.x[a] = fmaf(t, R.d[a], R.o[a]);
        P.site = cur = nearest_walk(&c->g, cur, P.x, &walk_steps);
        const float alpha = 1.f - expf(-cell_density(&c->g, &c->F, cur, P.x) * delta);
        const float w = T * alpha;
        const float T_after = T * (1.f - alpha);
        const int lit = w > c->w_thresh;
        if (lit) {
            blend_colour(&c->g, &c->F, &P, b);
            for (int ch = 0; ch < 3; ++ch) acc[ch] += w * P.C[ch];
        }
        float g_sigma = 0.f, g_colour[3];
        for (int ch = 0; ch < 3; ++ch) {
            g_sigma += gR[ch] * (T_after * P.C[ch] - (fg[ch] - acc[ch]));
            g_colour[ch] = lit ? w * gR[ch] : 0.f;
        }
        stop_grads(&c->g, &c->F, &P, delta * (g_sigma - tail), g_colour, b, &c->G);
        T = T_after;
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

/* Rotation of a unit quaternion (w, x, y, z) from its pairwise products (vgf.cu:340-344). */
static void rotation(const float u[4], float R[9]) {
    const float w = u[0], x = u[1], y = u[2], z = u[3];
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    const float rows[9] = {1.f - 2.f * (yy + zz), 2.f * (xy - wz), 2.f * (xz + wy),
                           2.f * (xy + wz), 1.f - 2.f * (xx + zz), 2.f * (yz - wx),
                           2.f * (xz - wy), 2.f * (yz + wx), 1.f - 2.f * (xx + yy)};
    memcpy(R, rows, sizeof(rows));
}

/* dL/dq from P = dL/dR of the rotation of q / |q|: P contracted with the partial derivatives of the
 * entries of rotation() with respect to (w, x, y, z), then the radial part removed and divided by |q|. */
static void quat_grad(const float u[4], float len, const float P[9], float g[4]) {
    const float w = u[0], x = u[1], y = u[2], z = u[3];
    const float J[4][9] = {
        {0.f, -2.f * z, 2.f * y, 2.f * z, 0.f, -2.f * x, -2.f * y, 2.f * x, 0.f},          /* d/dw */
        {0.f, 2.f * y, 2.f * z, 2.f * y, -4.f * x, -2.f * w, 2.f * z, 2.f * w, -4.f * x},  /* d/dx */
        {-4.f * y, 2.f * x, 2.f * w, 2.f * x, 0.f, 2.f * z, -2.f * w, 2.f * z, -4.f * y},  /* d/dy */
        {-4.f * z, -2.f * w, 2.f * x, 2.f * w, -4.f * z, 2.f * y, 2.f * x, 2.f * y, 0.f}}; /* d/dz */
    float raw[4], radial = 0.f;
    for (int c = 0; c < 4; ++c) {
        raw[c] = 0.f;
        for (int e = 0; e < 9; ++e) raw[c] += P[e] * J[c][e];
        radial += raw[c] * u[c];
    }
    for (int c = 0; c < 4; ++c) g[c] = (raw[c] - radial * u[c]) / len;
}

/* unit quaternion of row i and its length (at least 1e-12) */
static float unit_quat(const float* quat, int64_t i, float u[4]) {
    const float* q = quat + 4 * i;
    float sq = 0.f;
    for (int c = 0; c < 4; ++c) sq += q[c] * q[c];
    const float len = fmaxf(sqrtf(sq), 1e-12f);
    for (int c = 0; c < 4; ++c) u[c] = q[c] / len;
    return len;
}

typedef struct {
    float u[4], len, R[9], iv[3], s2[3];
} ConicSite;

/* R, s^2 = exp(2 clamp(ls, -20, 20)) and 1 / (s^2 + floor^2) of site i (vgf.cu:350-362) */
static void conic_site(const float* ls, const float* quat, int64_t i, float floor2, ConicSite* L) {
    L->len = unit_quat(quat, i, L->u);
    rotation(L->u, L->R);
    for (int k = 0; k < 3; ++k) {
        L->s2[k] = expf(2.f * fminf(fmaxf(ls[3 * i + k], -20.f), 20.f));
        L->iv[k] = 1.f / (L->s2[k] + floor2);
    }
}

static const int SYM_ROW[6] = {0, 0, 0, 1, 1, 2}, SYM_COL[6] = {0, 1, 2, 1, 2, 2};

/* A = R diag(iv) R^T in storage order (xx, xy, xz, yy, yz, zz) (vgf.cu:364-380) */
void vgo_conic_forward(const float* ls, const float* quat, int64_t n, float floor, float* A) {
    for (int64_t i = 0; i < n; ++i) {
        ConicSite L;
        conic_site(ls, quat, i, floor * floor, &L);
        for (int e = 0; e < 6; ++e) {
            const float* ra = L.R + 3 * SYM_ROW[e];
            const float* rb = L.R + 3 * SYM_COL[e];
            float sum = 0.f;
            for (int k = 0; k < 3; ++k) sum += ra[k] * L.iv[k] * rb[k];
            A[6 * i + e] = sum;
        }
    }
}

/* dL/dls and dL/dq from dL/dA (vgf.cu:382-421): with G the symmetric matrix of dL/dA,
 * dL/d iv_k = (R^T G R)_kk, d iv_k / d ls_k = -2 s_k^2 iv_k^2, dL/dR = 2 G R diag(iv). */
void vgo_conic_backward(const float* ls, const float* quat, int64_t n, float floor, const float* gA, float* g_ls,
                        float* g_quat) {
    for (int64_t i = 0; i < n; ++i) {
        ConicSite L;
        conic_site(ls, quat, i, floor * floor, &L);
        float G[9];
        for (int e = 0; e < 6; ++e) {
            const float v = SYM_ROW[e] == SYM_COL[e] ? gA[6 * i + e] : 0.5f * gA[6 * i + e];
            G[3 * SYM_ROW[e] + SYM_COL[e]] = G[3 * SYM_COL[e] + SYM_ROW[e]] = v;
        }
        float P[9];
        for (int k = 0; k < 3; ++k) {
            float diag = 0.f;
            for (int a = 0; a < 3; ++a) {
                float gr = 0.f; /* (G R)_ak */
                for (int m = 0; m < 3; ++m) gr += G[3 * a + m] * L.R[3 * m + k];
                diag += L.R[3 * a + k] * gr;
                P[3 * a + k] = 2.f * gr * L.iv[k];
            }
            g_ls[3 * i + k] = diag * (-2.f * L.s2[k] * L.iv[k] * L.iv[k]);
        }
        quat_grad(L.u, L.len, P, g_quat + 4 * i);
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

/* One site's Gaussian seen from x, its rotation rebuilt from the quaternion as the reference's field
 * kernels do (vgf.cu:99-124): v = x - p, y = R^T v, 1 / s_k^2 scaled by 1 / scale_mult^2, and the
 * Mahalanobis distance m = sum_k y_k^2 / s_k^2. */
typedef struct {
    float v[3], y[3], is2[3], u[4], len, R[9], m;
} SiteGauss;

static void site_gauss(const float* points, const float* ls, const float* quat, int i, const float x[3],
                       float inv_mult2, SiteGauss* L) {
    offset_to(points, i, x, L->v);
    L->len = unit_quat(quat, i, L->u);
    rotation(L->u, L->R);
    L->m = 0.f;
    for (int k = 0; k < 3; ++k) {
        L->y[k] = L->R[k] * L->v[0] + L->R[3 + k] * L->v[1] + L->R[6 + k] * L->v[2];
        const float s = expf(fminf(fmaxf(ls[3 * (int64_t)i + k], -20.f), 20.f));
        L->is2[k] = inv_mult2 / (s * s);
        L->m += L->y[k] * L->y[k] * L->is2[k];
    }
}

/* accumulates dL/dls and dL/dq of site i from gm = dL/dm (vgf.cu:126-153): dm/dls_k = -2 y_k^2 / s_k^2,
 * dL/dR_ab = v_a 2 gm y_b / s_b^2 */
static void site_gauss_grad(const SiteGauss* L, float gm, int i, float* g_ls, float* g_quat) {
    float scaled[3], P[9], gq[4];
    for (int k = 0; k < 3; ++k) {
        scaled[k] = 2.f * gm * L->y[k] * L->is2[k];
        g_ls[3 * (int64_t)i + k] += -2.f * gm * L->y[k] * L->y[k] * L->is2[k];
    }
    for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) P[3 * a + b] = L->v[a] * scaled[b];
    quat_grad(L->u, L->len, P, gq);
    for (int c = 0; c < 4; ++c) g_quat[4 * (int64_t)i + c] += gq[c];
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
            SiteGauss L;
            site_gauss(points, ls, quat, k, x + 3 * t, inv_mult2, &L);
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
            SiteGauss L;
            site_gauss(points, ls, quat, k, x + 3 * t, 1.f, &L);
            const float c = expf(fminf(raw[k], 30.f) - 0.5f * L.m);
            if (c * fabsf(gs) > 1e-12f) {
                g_raw[k] += gs * c;
                site_gauss_grad(&L, -0.5f * gs * c, k, g_ls, g_quat);
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

/* C(x, d) = sum_k a_k max(SH_k(d) + 1/2, 0) / sum_k a_k, a_k = exp(-(m_k - m_min) / 2), in one pass
 * with the sums rescaled whenever a smaller m arrives (vgf.cu:248-282) */
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
        float m_low = KINF, wsum = 0.f, sum[3] = {0.f, 0.f, 0.f};
        for (int j = 0; j < offsets[i + 1] - offsets[i] + 1; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            SiteGauss L;
            site_gauss(points, ls, quat, k, x + 3 * t, 1.f, &L);
            if (L.m < m_low) {
                const float shrink = m_low == KINF ? 0.f : expf(-0.5f * (m_low - L.m));
                wsum *= shrink;
                for (int ch = 0; ch < 3; ++ch) sum[ch] *= shrink;
                m_low = L.m;
            }
            const float a = expf(-0.5f * (L.m - m_low));
            float c[3];
            sh_eval(sh, k, b, nb, c);
            wsum += a;
            for (int ch = 0; ch < 3; ++ch) sum[ch] += a * fmaxf(c[ch], 0.f);
        }
        for (int ch = 0; ch < 3; ++ch) rgb[3 * t + ch] = sum[ch] / wsum;
    }
    return 0;
}

/* gradients of the blend, accumulated into zero-filled outputs (vgf.cu:284-335): dL/dsh_k = a_k b [c_k > 0]
 * gR, dL/dm_k = -a_k (gR . max(c_k, 0) - gR . C) / 2 */
int vgo_color_backward(const float* points, const int32_t* offsets, const int32_t* adj, int64_t n_sites,
                       const float* ls, const float* quat, const float* sh, int sh_deg, const float* x,
                       const float* dirs, const int32_t* site, int64_t m, const float* rgb, const float* grad_rgb,
                       float* g_ls, float* g_quat, float* g_sh) {
    (void)n_sites;
    const int nb = (sh_deg + 1) * (sh_deg + 1);
    for (int64_t t = 0; t < m; ++t) {
        const float* gR = grad_rgb + 3 * t;
        if (gR[0] == 0.f && gR[1] == 0.f && gR[2] == 0.f) continue;
        const int i = site[t], n = offsets[i + 1] - offsets[i] + 1;
        float m_low = KINF, wsum = 0.f;
        for (int j = 0; j < n; ++j) {
            SiteGauss L;
            site_gauss(points, ls, quat, nbhd(offsets, adj, i, j), x + 3 * t, 1.f, &L);
            m_low = fminf(m_low, L.m);
        }
        for (int j = 0; j < n; ++j) {
            SiteGauss L;
            site_gauss(points, ls, quat, nbhd(offsets, adj, i, j), x + 3 * t, 1.f, &L);
            wsum += expf(-0.5f * (L.m - m_low));
        }
        const float inv_sum = 1.f / wsum;
        const float gRC = dot3(gR, rgb + 3 * t);
        float d[3], b[16];
        unit_dir(dirs, t, d);
        sh_basis(d[0], d[1], d[2], sh_deg, b);
        for (int j = 0; j < n; ++j) {
            const int k = nbhd(offsets, adj, i, j);
            SiteGauss L;
            site_gauss(points, ls, quat, k, x + 3 * t, 1.f, &L);
            const float a = expf(-0.5f * (L.m - m_low)) * inv_sum;
            if (a < MIN_WEIGHT) continue;
            float c[3], dc[3];
            sh_eval(sh, k, b, nb, c);
            for (int ch = 0; ch < 3; ++ch) dc[ch] = c[ch] > 0.f ? a * gR[ch] : 0.f;
            float* gs = g_sh + 48 * (int64_t)k;
            for (int q = 0; q < nb; ++q)
                for (int ch = 0; ch < 3; ++ch) gs[3 * q + ch] += b[q] * dc[ch];
            const float gm = -0.5f * a * (dot3_pos(gR, c) - gRC);
            if (gm != 0.f) site_gauss_grad(&L, gm, k, g_ls, g_quat);
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
