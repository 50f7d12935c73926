/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the arithmetic behind the reference's hot path.
 * The reference's contract (official/reference.py:125-127 `ref_kernel`,
 * submissions/baseline_geqrf.py:5-6) is `torch.geqrf(A)`, i.e. LAPACK
 * xGEQRF: batched square Householder QR returned in compact form
 * (R on/above the diagonal, Householder vectors below it, plus tau).
 * LAPACK is a third-party dependency of the reference (pinned through the
 * installed torch wheel: MKL 2024.2 on CPU); its published algorithm
 * (xGEQR2 / xLARFG / xLARF, xORG2R, and the compact-WY xLARFT/xLARFB pair)
 * is restated here from the mathematics, in our own code.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker.  Nothing in the product path
 * links or calls it.
 *
 * Storage conventions used by every function below:
 *   - input A: float32, element (i, j) of matrix b at
 *       A[b*a_bs + i*a_rs + j*a_cs]   (the reference passes row-major
 *       contiguous tensors, official/reference.py:142, i.e. a_rs=n, a_cs=1)
 *   - output H: column-major n x n per matrix, element (i, j) at
 *       H[b*n*n + j*n + i]  (torch.geqrf's (n*n, 1, n) strides, which the
 *       reference's candidate also returns, submissions/candidate.py:3752-3769)
 *   - tau: [batch][n] contiguous.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_EINVAL 1
#define ORACLE_ENOMEM 2

/* ---------------------------------------------------------------------- */
/* Reflector generation, xLARFG semantics.                                */
/*                                                                        */
/* Given alpha and x (length m), find beta, tau, v with v(0)=1 such that  */
/* (I - tau v v^T) [alpha; x] = [beta; 0].  If ||x|| == 0 then tau = 0    */
/* and nothing changes (H = I).  Otherwise                                */
/*   beta = -sign(alpha) * hypot(alpha, ||x||)                            */
/*   tau  = (beta - alpha) / beta                                         */
/*   x   := x / (alpha - beta)                                            */
/* The norm is accumulated in double (long double for the double path) so */
/* that no finite float input can overflow or underflow it.               */
/* ---------------------------------------------------------------------- */
static double larfg_d(int64_t m, double *alpha, double *x, int64_t incx)
{
    long double ss = 0.0L;
    for (int64_t i = 0; i < m; ++i) {
        long double xi = (long double)x[i * incx];
        ss += xi * xi;
    }
    if (ss == 0.0L) return 0.0;
    long double a = (long double)(*alpha);
    long double r = sqrtl(a * a + ss);
    double beta = (double)(signbit((double)a) ? r : -r);
    double tau = (beta - *alpha) / beta;
    double scale = 1.0 / (*alpha - beta);
    for (int64_t i = 0; i < m; ++i) x[i * incx] *= scale;
    *alpha = beta;
    return tau;
}

static float larfg_f(int64_t m, float *alpha, float *x, int64_t incx)
{
    double ss = 0.0;
    for (int64_t i = 0; i < m; ++i) {
        double xi = (double)x[i * incx];
        ss += xi * xi;
    }
    if (ss == 0.0) return 0.0f;
    double a = (double)(*alpha);
    double r = sqrt(a * a + ss);
    float beta = (float)(signbit(a) ? r : -r);
    float tau = (beta - *alpha) / beta;
    float scale = 1.0f / (*alpha - beta);
    for (int64_t i = 0; i < m; ++i) x[i * incx] *= scale;
    *alpha = beta;
    return tau;
}

/* ---------------------------------------------------------------------- */
/* Unblocked QR of one column-major m x n matrix (lda >= m), xGEQR2.      */
/* For each column k: generate H_k from a(k:m, k), then apply H_k from the */
/* left to a(k:m, k+1:n):  w = a^T v,  a -= tau v w^T.                    */
/* ---------------------------------------------------------------------- */
static void geqr2_d(int64_t m, int64_t n, double *a, int64_t lda, double *tau, double *work)
{
    int64_t kmax = m < n ? m : n;
    for (int64_t k = 0; k < kmax; ++k) {
        double *col = a + k * lda;
        double t = larfg_d(m - k - 1, &col[k], col + k + 1, 1);
        tau[k] = t;
        if (t == 0.0) continue;
        double akk = col[k];
        col[k] = 1.0;
        for (int64_t j = k + 1; j < n; ++j) {
            const double *cj = a + j * lda;
            double w = 0.0;
            for (int64_t i = k; i < m; ++i) w += col[i] * cj[i];
            work[j] = w;
        }
        for (int64_t j = k + 1; j < n; ++j) {
            double *cj = a + j * lda;
            double tw = t * work[j];
            for (int64_t i = k; i < m; ++i) cj[i] -= col[i] * tw;
        }
        col[k] = akk;
    }
    for (int64_t k = kmax; k < n; ++k) tau[k] = 0.0;
}

static void geqr2_f(int64_t m, int64_t n, float *a, int64_t lda, float *tau, float *work)
{
    int64_t kmax = m < n ? m : n;
    for (int64_t k = 0; k < kmax; ++k) {
        float *col = a + k * lda;
        float t = larfg_f(m - k - 1, &col[k], col + k + 1, 1);
        tau[k] = t;
        if (t == 0.0f) continue;
        float akk = col[k];
        col[k] = 1.0f;
        for (int64_t j = k + 1; j < n; ++j) {
            const float *cj = a + j * lda;
            float w = 0.0f;
            for (int64_t i = k; i < m; ++i) w += col[i] * cj[i];
            work[j] = w;
        }
        for (int64_t j = k + 1; j < n; ++j) {
            float *cj = a + j * lda;
            float tw = t * work[j];
            for (int64_t i = k; i < m; ++i) cj[i] -= col[i] * tw;
        }
        col[k] = akk;
    }
    for (int64_t k = kmax; k < n; ++k) tau[k] = 0.0f;
}

static int check_args(int64_t batch, int64_t n, const float *A, const void *H, const void *tau)
{
    if (batch < 0 || n < 0) return ORACLE_EINVAL;
    if (batch > 0 && n > 0 && (!A || !H || !tau)) return ORACLE_EINVAL;
    return ORACLE_OK;
}

/* Batched geqrf in double arithmetic: H, tau are float64. */
int oracle_geqrf_f64(int64_t batch, int64_t n, const float *A, int64_t a_bs, int64_t a_rs,
                     int64_t a_cs, double *H, double *tau)
{
    int rc = check_args(batch, n, A, H, tau);
    if (rc) return rc;
    double *work = (double *)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    if (!work) return ORACLE_ENOMEM;
    for (int64_t b = 0; b < batch; ++b) {
        double *h = H + b * n * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < n; ++i) h[j * n + i] = (double)A[b * a_bs + i * a_rs + j * a_cs];
        geqr2_d(n, n, h, n, tau + b * n, work);
    }
    free(work);
    return ORACLE_OK;
}

/* Batched geqrf in float arithmetic (norms in double): H, tau are float32. */
int oracle_geqrf_f32(int64_t batch, int64_t n, const float *A, int64_t a_bs, int64_t a_rs,
                     int64_t a_cs, float *H, float *tau)
{
    int rc = check_args(batch, n, A, H, tau);
    if (rc) return rc;
    float *work = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    if (!work) return ORACLE_ENOMEM;
    for (int64_t b = 0; b < batch; ++b) {
        float *h = H + b * n * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < n; ++i) h[j * n + i] = A[b * a_bs + i * a_rs + j * a_cs];
        geqr2_f(n, n, h, n, tau + b * n, work);
    }
    free(work);
    return ORACLE_OK;
}

/* Batched geqrf of m x n matrices (any m, n) in double arithmetic, the   */
/* same xGEQR2 steps (min(m, n) reflectors): H is column-major m x n per  */
/* matrix (float64), tau holds min(m, n) values per matrix.               */
int oracle_geqrf_rect_f64(int64_t batch, int64_t m, int64_t n, const float *A, int64_t a_bs,
                          int64_t a_rs, int64_t a_cs, double *H, double *tau)
{
    if (batch < 0 || m < 0 || n < 0) return ORACLE_EINVAL;
    if (batch > 0 && m > 0 && n > 0 && (!A || !H || !tau)) return ORACLE_EINVAL;
    const int64_t kmax = m < n ? m : n;
    double *work = (double *)malloc(sizeof(double) * (size_t)(2 * n + 1));
    if (!work) return ORACLE_ENOMEM;
    double *tk = work + n;  /* geqr2_d writes n tau values */
    for (int64_t b = 0; b < batch; ++b) {
        double *h = H + b * m * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < m; ++i) h[j * m + i] = (double)A[b * a_bs + i * a_rs + j * a_cs];
        geqr2_d(m, n, h, m > 0 ? m : 1, tk, work);
        for (int64_t k = 0; k < kmax; ++k) tau[b * kmax + k] = tk[k];
    }
    free(work);
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Blocked compact-WY QR, double arithmetic.  The panel algorithm of      */
/* tools/blocked_qr_reference.py:192-262 (update_mode="compact-wy"):      */
/* factor the m x nb panel with geqr2, form the upper-triangular T with   */
/*   T(j,j) = tau_j,  T(0:j, j) = -tau_j T(0:j,0:j) V(:,0:j)^T v_j        */
/* (tools/blocked_qr_reference.py:98-109), then update the trailing block */
/*   C := C - V ( T^T ( V^T C ) )                                         */
/* (tools/blocked_qr_reference.py:112-122).  This is the algorithm the    */
/* GPU's blocked path executes; it is compared with geqr2 in the tests.   */
/* ---------------------------------------------------------------------- */
int oracle_geqrf_blocked_f64(int64_t batch, int64_t n, int64_t nb, const float *A, int64_t a_bs,
                             int64_t a_rs, int64_t a_cs, double *H, double *tau)
{
    int rc = check_args(batch, n, A, H, tau);
    if (rc) return rc;
    if (nb <= 0) return ORACLE_EINVAL;
    size_t nn = (size_t)(n > 0 ? n : 1);
    double *work = (double *)malloc(sizeof(double) * nn);
    double *T = (double *)malloc(sizeof(double) * (size_t)nb * (size_t)nb);
    double *W = (double *)malloc(sizeof(double) * (size_t)nb * nn);
    double *Y = (double *)malloc(sizeof(double) * (size_t)nb * nn);
    double *V = (double *)malloc(sizeof(double) * (size_t)nb * nn);
    if (!work || !T || !W || !Y || !V) {
        free(work); free(T); free(W); free(Y); free(V);
        return ORACLE_ENOMEM;
    }
    for (int64_t b = 0; b < batch; ++b) {
        double *h = H + b * n * n;
        double *tb = tau + b * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < n; ++i) h[j * n + i] = (double)A[b * a_bs + i * a_rs + j * a_cs];
        for (int64_t k = 0; k < n; k += nb) {
            int64_t w = nb < n - k ? nb : n - k;
            int64_t m = n - k;
            double *panel = h + k * n + k;
            geqr2_d(m, w, panel, n, tb + k, work);
            int64_t nc = n - k - w;
            if (nc <= 0) continue;
            /* V: m x w, unit lower trapezoidal, column-major with ld m */
            for (int64_t j = 0; j < w; ++j)
                for (int64_t i = 0; i < m; ++i)
                    V[j * m + i] = i < j ? 0.0 : (i == j ? 1.0 : panel[j * n + i]);
            /* T: w x w upper triangular, column-major */
            memset(T, 0, sizeof(double) * (size_t)(w * w));
            for (int64_t j = 0; j < w; ++j) {
                double tj = tb[k + j];
                T[j * w + j] = tj;
                for (int64_t i = 0; i < j; ++i) {
                    double y = 0.0;
                    for (int64_t r = 0; r < m; ++r) y += V[i * m + r] * V[j * m + r];
                    work[i] = -tj * y;
                }
                for (int64_t i = 0; i < j; ++i) {
                    double s = 0.0;
                    for (int64_t l = i; l < j; ++l) s += T[l * w + i] * work[l];
                    T[j * w + i] = s;
                }
            }
            /* W = V^T C  (w x nc) */
            double *C = h + (k + w) * n + k;
            for (int64_t c = 0; c < nc; ++c)
                for (int64_t j = 0; j < w; ++j) {
                    double s = 0.0;
                    for (int64_t r = 0; r < m; ++r) s += V[j * m + r] * C[c * n + r];
                    W[c * w + j] = s;
                }
            /* Y = T^T W */
            for (int64_t c = 0; c < nc; ++c)
                for (int64_t j = 0; j < w; ++j) {
                    double s = 0.0;
                    for (int64_t l = 0; l <= j; ++l) s += T[j * w + l] * W[c * w + l];
                    Y[c * w + j] = s;
                }
            /* C -= V Y */
            for (int64_t c = 0; c < nc; ++c)
                for (int64_t j = 0; j < w; ++j) {
                    double y = Y[c * w + j];
                    for (int64_t r = j; r < m; ++r) C[c * n + r] -= V[j * m + r] * y;
                }
        }
    }
    free(work); free(T); free(W); free(Y); free(V);
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Q from compact (H, tau), LAPACK xORG2R / torch.linalg.householder_product */
/* (used by the official checker, official/reference.py:199).             */
/* Q = H_0 H_1 ... H_{n-1} applied to I, accumulated backwards.            */
/* H is column-major n x n per matrix; Q is written column-major.         */
/* ---------------------------------------------------------------------- */
int oracle_orgqr_f64(int64_t batch, int64_t n, const float *H, const float *tau, double *Q)
{
    if (batch < 0 || n < 0) return ORACLE_EINVAL;
    double *v = (double *)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    if (!v) return ORACLE_ENOMEM;
    for (int64_t b = 0; b < batch; ++b) {
        const float *h = H + b * n * n;
        const float *t = tau + b * n;
        double *q = Q + b * n * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < n; ++i) q[j * n + i] = i == j ? 1.0 : 0.0;
        for (int64_t k = n - 1; k >= 0; --k) {
            double tk = (double)t[k];
            if (tk == 0.0) continue;
            v[k] = 1.0;
            for (int64_t i = k + 1; i < n; ++i) v[i] = (double)h[k * n + i];
            for (int64_t j = k; j < n; ++j) {
                double *qj = q + j * n;
                double s = 0.0;
                for (int64_t i = k; i < n; ++i) s += v[i] * qj[i];
                s *= tk;
                for (int64_t i = k; i < n; ++i) qj[i] -= v[i] * s;
            }
        }
    }
    free(v);
    return ORACLE_OK;
}

/* Same product accumulated in float arithmetic, as
 * torch.linalg.householder_product does on float32 inputs. */
int oracle_orgqr_f32(int64_t batch, int64_t n, const float *H, const float *tau, float *Q)
{
    if (batch < 0 || n < 0) return ORACLE_EINVAL;
    float *v = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    if (!v) return ORACLE_ENOMEM;
    for (int64_t b = 0; b < batch; ++b) {
        const float *h = H + b * n * n;
        const float *t = tau + b * n;
        float *q = Q + b * n * n;
        for (int64_t j = 0; j < n; ++j)
            for (int64_t i = 0; i < n; ++i) q[j * n + i] = i == j ? 1.0f : 0.0f;
        for (int64_t k = n - 1; k >= 0; --k) {
            float tk = t[k];
            if (tk == 0.0f) continue;
            v[k] = 1.0f;
            for (int64_t i = k + 1; i < n; ++i) v[i] = h[k * n + i];
            for (int64_t j = k; j < n; ++j) {
                float *qj = q + j * n;
                float s = 0.0f;
                for (int64_t i = k; i < n; ++i) s += v[i] * qj[i];
                s *= tk;
                for (int64_t i = k; i < n; ++i) qj[i] -= v[i] * s;
            }
        }
    }
    free(v);
    return ORACLE_OK;
}

const char *oracle_version(void) { return "fastqr-oracle 1"; }
