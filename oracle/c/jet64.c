/*
 * FP64 C restatement of the fixed 2 -> 64x4 -> 1 tanh MLP forward-Laplacian jet and of its
 * hand-derived adjoint (TEST INFRASTRUCTURE ONLY: built into oracle/_build/ and loaded by
 * the tests as an independent checker; never linked into the shipped library).
 *
 * Parameter layout: the packed ABI of csrc/mlp_abi.cuh:8-17 (reference), i.e. per layer
 * W[out][in] row-major followed by b[out]; offsets 0/128/192/4288/4352/8448/8512/12608/
 * 12672/12736, 12,737 values in total.
 *
 * Forward jet (reference csrc/fused_residual.cu:16-23, :79-117):
 *   linear: z_v = W v + b, z_J = W J, z_L = W L; layer 0 has J = W0 and L = 0
 *   tanh:   a = tanh(z_v), s = 1 - a^2
 *           v = a, J = s z_J, L = s z_L - 2 a s (z_J0^2 + z_J1^2)
 *   output: u = w.v + b, lap = w.L
 * Adjoint of tanh (reference csrc/fused_backward.cu:29-33, :75-89), with s2 = -2 a s,
 * s3 = -2 s^2 + 4 a^2 s, q = z_J0^2 + z_J1^2:
 *   zbar_v  = vbar s + (Jbar . z_J) s2 + Lbar (z_L s2 + q s3)
 *   zbar_Jd = Jbar_d s + 2 Lbar s2 z_Jd
 *   zbar_L  = Lbar s
 * Layer 0 (reference csrc/fused_backward.cu:337-359):
 *   db0 = zbar_v, dW0[o][d] = zbar_v x_d + zbar_Jd, dx_d = sum_o W0[o][d] zbar_v
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { IN = 2, H = 64, LAYERS = 4, NPARAM = 12737 };
enum { B0 = H * IN, HBASE = B0 + H, HSTRIDE = H * H + H, OUTBASE = HBASE + 3 * HSTRIDE };

typedef struct {
  double z[LAYERS][4][H]; /* pre-activation jets, components v, J0, J1, L */
  double h[LAYERS][4][H]; /* post-activation jets */
} Tape;

static void tanh_forward(const double *z, double *h, int o) {
  const double zv = z[0 * H + o], zj0 = z[1 * H + o], zj1 = z[2 * H + o], zl = z[3 * H + o];
  const double a = tanh(zv);
  const double s = 1.0 - a * a;
  h[0 * H + o] = a;
  h[1 * H + o] = s * zj0;
  h[2 * H + o] = s * zj1;
  h[3 * H + o] = s * zl - 2.0 * a * s * (zj0 * zj0 + zj1 * zj1);
}

static void forward_point(const double *p, double x0, double x1, Tape *t, double *u,
                          double *lap) {
  for (int o = 0; o < H; ++o) {
    const double w0 = p[o * IN], w1 = p[o * IN + 1];
    t->z[0][0][o] = w0 * x0 + w1 * x1 + p[B0 + o];
    t->z[0][1][o] = w0;
    t->z[0][2][o] = w1;
    t->z[0][3][o] = 0.0;
    tanh_forward(&t->z[0][0][0], &t->h[0][0][0], o);
  }
  for (int l = 1; l < LAYERS; ++l) {
    const double *w = p + HBASE + (l - 1) * HSTRIDE;
    const double *b = w + H * H;
    for (int o = 0; o < H; ++o) {
      for (int c = 0; c < 4; ++c) {
        double acc = c == 0 ? b[o] : 0.0;
        for (int i = 0; i < H; ++i) acc += w[o * H + i] * t->h[l - 1][c][i];
        t->z[l][c][o] = acc;
      }
      tanh_forward(&t->z[l][0][0], &t->h[l][0][0], o);
    }
  }
  const double *wo = p + OUTBASE;
  double uu = wo[H], ll = 0.0;
  for (int i = 0; i < H; ++i) {
    uu += wo[i] * t->h[LAYERS - 1][0][i];
    ll += wo[i] * t->h[LAYERS - 1][3][i];
  }
  *u = uu;
  *lap = ll;
}

void jet64_forward(const double *params, const double *xy, int64_t n, double *u, double *lap) {
  Tape t;
  for (int64_t k = 0; k < n; ++k) forward_point(params, xy[2 * k], xy[2 * k + 1], &t, u + k, lap + k);
}

/* adj holds hbar on entry and zbar on exit for every neuron of one layer */
static void tanh_backward(const double z[4][H], double adj[4][H]) {
  for (int o = 0; o < H; ++o) {
    const double zv = z[0][o], zj0 = z[1][o], zj1 = z[2][o], zl = z[3][o];
    const double a = tanh(zv);
    const double s = 1.0 - a * a;
    const double s2 = -2.0 * a * s;
    const double s3 = -2.0 * s * s + 4.0 * a * a * s;
    const double q = zj0 * zj0 + zj1 * zj1;
    const double av = adj[0][o], aj0 = adj[1][o], aj1 = adj[2][o], al = adj[3][o];
    adj[0][o] = av * s + (aj0 * zj0 + aj1 * zj1) * s2 + al * (zl * s2 + q * s3);
    adj[1][o] = aj0 * s + 2.0 * al * s2 * zj0;
    adj[2][o] = aj1 * s + 2.0 * al * s2 * zj1;
    adj[3][o] = al * s;
  }
}

void jet64_backward(const double *params, const double *xy, const double *grad_u,
                    const double *grad_lap, int64_t n, double *grad_params, double *grad_xy) {
  Tape t;
  double adj[4][H], prev[4][H];
  memset(grad_params, 0, sizeof(double) * NPARAM);
  const double *wo = params + OUTBASE;
  for (int64_t k = 0; k < n; ++k) {
    const double x0 = xy[2 * k], x1 = xy[2 * k + 1], gu = grad_u[k], gl = grad_lap[k];
    double u, lap;
    forward_point(params, x0, x1, &t, &u, &lap);
    /* output layer: u = w.v + b, lap = w.L */
    for (int i = 0; i < H; ++i) {
      grad_params[OUTBASE + i] += gu * t.h[LAYERS - 1][0][i] + gl * t.h[LAYERS - 1][3][i];
      adj[0][i] = gu * wo[i];
      adj[1][i] = 0.0;
      adj[2][i] = 0.0;
      adj[3][i] = gl * wo[i];
    }
    grad_params[OUTBASE + H] += gu;
    for (int l = LAYERS - 1; l >= 1; --l) {
      const double *w = params + HBASE + (l - 1) * HSTRIDE;
      double *gw = grad_params + HBASE + (l - 1) * HSTRIDE;
      tanh_backward(t.z[l], adj);
      for (int o = 0; o < H; ++o) {
        gw[H * H + o] += adj[0][o];
        for (int i = 0; i < H; ++i) {
          double acc = 0.0;
          for (int c = 0; c < 4; ++c) acc += adj[c][o] * t.h[l - 1][c][i];
          gw[o * H + i] += acc;
        }
      }
      for (int c = 0; c < 4; ++c)
        for (int i = 0; i < H; ++i) {
          double acc = 0.0;
          for (int o = 0; o < H; ++o) acc += w[o * H + i] * adj[c][o];
          prev[c][i] = acc;
        }
      memcpy(adj, prev, sizeof(adj));
    }
    tanh_backward(t.z[0], adj);
    double gx0 = 0.0, gx1 = 0.0;
    for (int o = 0; o < H; ++o) {
      grad_params[B0 + o] += adj[0][o];
      grad_params[o * IN] += adj[0][o] * x0 + adj[1][o];
      grad_params[o * IN + 1] += adj[0][o] * x1 + adj[2][o];
      gx0 += params[o * IN] * adj[0][o];
      gx1 += params[o * IN + 1] * adj[0][o];
    }
    grad_xy[2 * k] = gx0;
    grad_xy[2 * k + 1] = gx1;
  }
}

int jet64_parameter_count(void) { return NPARAM; }
