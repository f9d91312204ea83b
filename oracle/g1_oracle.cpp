// CPU oracle of the G1 control step: a scalar restatement, in float64 (or float32), of the algorithm the reference
// runs on the GPU. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and bench.py's CPU-baseline leg call it
// as the checker; the product path (nablaengine_b200) never links or calls it.
//
// What it restates, step by step (reference = OamIcs/NablaEngine, paths under its repository):
//   smooth dynamics   src/nablaengine/g1_engine/source.py:102-334 (fwd_body, body_force, body_inertia, torques):
//                     forward kinematics, bias forces by Newton-Euler with qacc = 0 (gravity as a base
//                     acceleration), the joint-space mass matrix plus armature; written here as sums over bodies of
//                     J' m J and Jr' I Jr (the same matrix as the reference's composite-rigid-body recursion)
//   actuation         step.py:1762-1778: PD force kp (ctrl - q) - kv qdot clamped to the joint's actuator force range
//   collision         step.py:436-556, 1043-1145: plane-sphere, plane-capsule (both ends, frame along the projected
//                     axis), sphere-sphere, sphere-capsule (regularised segment point), capsule-capsule (clamp
//                     cascade; the parallel case's end candidates); MuJoCo's make_frame
//   constraint rows   step.py:1881-1957, 1147-1188: hinge-limit rows, pyramidal rows n +- mu t1, n +- mu t2 for
//                     condim 3, one normal row for condim 1; refsafe impedance, diagonal approximation from
//                     invweight0, D = 1 / R, aref = -b v - k imp pos; capacity 64 contacts / 192 rows
//   Newton solver     step.py:1969-2137: warm start or qacc_smooth by total cost, Hessian M + J'DJ on the quadratic
//                     rows, Cholesky, exact line search (safeguarded 1-D Newton, <= 40 steps), stopping test
//                     improvement < tol or |grad| < tol scaled by 1 / (meaninertia nv)
//   implicitfast      step.py:2153-2182: (M + h kv) a_adv = M a*, qvel += h a_adv, qpos integrated with the new qvel
//                     (free joint: quaternion times exp(h w / 2), renormalised)
//   substep chaining  host.py:133-234: warm start of substep k is the solution of substep k - 1; info = [iterations
//                     of the last substep, its raw contact count, its rows, overflow bits ORed over the substeps]
// Contacts are ordered deterministically: pair order, then the pair's contact slot (MuJoCo's own order).
#include <algorithm>
#include <omp.h>
#include <cmath>
#include <cstring>
#include <vector>

#define NB_MODEL_CONST static const
#include "../nablaengine_b200/csrc/g1_model_data.h"

namespace {

constexpr int NQ = G1_NQ, NV = G1_NV, NU = G1_NU, NBODY = G1_NBODY, NGEOM = G1_NGEOM, NPAIR = G1_NPAIR;
constexpr int MAXCON = 64, NEFC = 192;

template <class T> struct V3 {
  T x[3];
  T& operator[](int i) { return x[i]; }
  const T& operator[](int i) const { return x[i]; }
};
template <class T> V3<T> v3(T a, T b, T c) { return V3<T>{{a, b, c}}; }
template <class T> V3<T> operator+(const V3<T>& a, const V3<T>& b) { return v3(a[0] + b[0], a[1] + b[1], a[2] + b[2]); }
template <class T> V3<T> operator-(const V3<T>& a, const V3<T>& b) { return v3(a[0] - b[0], a[1] - b[1], a[2] - b[2]); }
template <class T> V3<T> operator*(T s, const V3<T>& a) { return v3(s * a[0], s * a[1], s * a[2]); }
template <class T> T dot(const V3<T>& a, const V3<T>& b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }
template <class T> V3<T> cross(const V3<T>& a, const V3<T>& b) {
  return v3(a[1] * b[2] - a[2] * b[1], a[2] * b[0] - a[0] * b[2], a[0] * b[1] - a[1] * b[0]);
}
template <class T> struct Q4 { T w, x, y, z; };
template <class T> Q4<T> qmul(const Q4<T>& a, const Q4<T>& b) {
  return Q4<T>{a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z, a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
               a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x, a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
}
template <class T> V3<T> qrot(const Q4<T>& q, const V3<T>& v) {  // q v q^-1
  V3<T> u = v3(q.x, q.y, q.z);
  V3<T> t = T(2) * cross(u, v);
  return v + q.w * t + cross(u, t);
}
template <class T> V3<T> qrot_inv(const Q4<T>& q, const V3<T>& v) { return qrot(Q4<T>{q.w, -q.x, -q.y, -q.z}, v); }
template <class T> V3<T> mv3(const double* p) { return v3(T(p[0]), T(p[1]), T(p[2])); }
template <class T> Q4<T> mq4(const double* p) { return Q4<T>{T(p[0]), T(p[1]), T(p[2]), T(p[3])}; }

template <class T> struct Contact {
  int pair, slot;
  T dist, mu;
  V3<T> pos, frame[3];
};

// The adjoint's gradient modes other than the exact derivative (reference g1_engine/adjoint.py:38-57, the clamp
// options DK_ADJ_CLAMP_KV; g1_engine/adjoint_contact.py:76-90, the self-contact normal option DK_ADJ_NORMAL and the
// near-parallel capsule rule DK_ADJ_PARALLEL) are exact derivatives of a surrogate step that holds some quantities at
// their values on the base trajectory (the unperturbed step); central differences of the surrogate around the base
// state therefore check them. Per substep of the base trajectory, ModeBase keeps: the dofs whose actuator force is
// clamped, their input velocity and unclamped PD force, and for every contact of the sphere core (sphere-sphere,
// sphere-capsule, capsule-capsule) its normal, centre distance nu and segment parameters. The surrogate:
//  - clamp_kv 1 (exact): a clamped dof's force is its bound; 0: the bound minus kv (v - v_base) (the damping
//    derivative kept); 2: the bound plus w (f - f_base), w = exp(-max((|f_base| - lim) / lim, 0) / soft) (soft <= 0:
//    w = 0), f the unclamped PD force;
//  - normal 0: exact; otherwise the core's normal is n_base + s (n - n_base), s = 0 (1: frozen), nu_base /
//    max(nu_base, 1e-3) (2), nu_base < 1e-3 ? 0 : 1 (3), with the contact point and frame built from it; and a
//    capsule-capsule contact with both segment parameters free on axes with sin^2 < 1.2e-3 keeps the base's
//    parameters.
struct ModeContact { int pair, slot; double n[3], nu, x1, x2; bool hold; };
struct ModeBase {
  unsigned long long clamp = 0;
  double v[NV] = {}, f[NV] = {};
  std::vector<ModeContact> con;
};
struct Mode {
  int clamp_kv = 1, normal = 0;
  double soft = 0;
  bool record = false;        // the base pass: fill base[k]; else apply the surrogate with base[k]
  ModeBase* base = nullptr;   // (nsub)
  int k = 0;                  // the current substep
};

// one world's working state for one substep
template <class T> struct World {
  // inputs / state
  T qpos[NQ], qvel[NV], qacc[NV];
  const T* ctrl;
  T fric;
  V3<T> com;
  // kinematics
  Q4<T> xq[NBODY];
  V3<T> xpos[NBODY], xipos[NBODY], wax[NV], anchor[NV];  // dof axes (world) and the point they rotate about
  bool trans[NV];
  // dynamics
  T M[NV][NV], qfrc_smooth[NV], qacc_smooth[NV];
  // constraints
  std::vector<Contact<T>> con;
  int ncon_raw;
  int nrow;
  T J[NEFC][NV], D[NEFC], aref[NEFC];
  int unsupported;
  Mode* mode = nullptr;  // a gradient mode's base pass or surrogate (test infrastructure), or none
};

template <class T> bool is_ancestor_dof(int dof, int body) {  // dof belongs to body or to one of its ancestors
  int db = g1_dof_body[dof];
  for (int b = body; b > 0; b = g1_body_parent[b])
    if (b == db) return true;
  return false;
}

// world-frame velocity Jacobian column of dof i at point p (zero when dof i is not on p's body chain)
template <class T> V3<T> jac_point(const World<T>& w, int i, const V3<T>& p) {
  if (w.trans[i]) return w.wax[i];
  return cross(w.wax[i], p - w.anchor[i]);
}

template <class T> void kinematics(World<T>& w) {
  w.xq[0] = Q4<T>{1, 0, 0, 0};
  w.xpos[0] = v3<T>(0, 0, 0);
  w.xipos[0] = w.xpos[0];
  for (int b = 1; b < NBODY; b++) {
    if (b == 1) {
      T n = std::sqrt(w.qpos[3] * w.qpos[3] + w.qpos[4] * w.qpos[4] + w.qpos[5] * w.qpos[5] + w.qpos[6] * w.qpos[6]);
      w.xq[1] = Q4<T>{w.qpos[3] / n, w.qpos[4] / n, w.qpos[5] / n, w.qpos[6] / n};
      w.xpos[1] = v3(w.qpos[0], w.qpos[1], w.qpos[2]);
      for (int k = 0; k < 3; k++) {
        w.trans[k] = true;
        V3<T> e = v3<T>(0, 0, 0);
        e[k] = 1;
        w.wax[k] = e;
        w.anchor[k] = w.xpos[1];
        w.trans[3 + k] = false;
        w.wax[3 + k] = qrot(w.xq[1], e);  // the free joint's angular velocity is in the local frame
        w.anchor[3 + k] = w.xpos[1];
      }
    } else {
      int p = g1_body_parent[b];
      V3<T> ax = mv3<T>(g1_body_axis + 3 * b);
      T ang = w.qpos[g1_body_qposadr[b]];
      T s = std::sin(ang / 2), c = std::cos(ang / 2);
      Q4<T> q0 = qmul(w.xq[p], mq4<T>(g1_body_quat + 4 * b));
      w.xq[b] = qmul(q0, Q4<T>{c, s * ax[0], s * ax[1], s * ax[2]});
      w.xpos[b] = w.xpos[p] + qrot(w.xq[p], mv3<T>(g1_body_pos + 3 * b));
      int d = g1_body_dofadr[b];
      w.trans[d] = false;
      w.wax[d] = qrot(w.xq[b], ax);
      w.anchor[d] = w.xpos[b];
    }
    V3<T> ip = mv3<T>(g1_body_ipos + 3 * b);
    if (b == G1_TORSO) ip = ip + w.com;  // per-world torso COM offset
    w.xipos[b] = w.xpos[b] + qrot(w.xq[b], ip);
  }
}

// world inertia tensor of body b (3x3)
template <class T> void body_inertia_world(const World<T>& w, int b, T I[3][3]) {
  Q4<T> qi = qmul(w.xq[b], mq4<T>(g1_body_iquat + 4 * b));
  V3<T> col[3];
  for (int k = 0; k < 3; k++) {
    V3<T> e = v3<T>(0, 0, 0);
    e[k] = 1;
    col[k] = qrot(qi, e);
  }
  for (int r = 0; r < 3; r++)
    for (int c = 0; c < 3; c++) {
      T s = 0;
      for (int k = 0; k < 3; k++) s += col[k][r] * T(g1_body_inertia[3 * b + k]) * col[k][c];
      I[r][c] = s;
    }
}
template <class T> V3<T> mat3v(const T A[3][3], const V3<T>& v) {
  return v3(A[0][0] * v[0] + A[0][1] * v[1] + A[0][2] * v[2], A[1][0] * v[0] + A[1][1] * v[1] + A[1][2] * v[2],
            A[2][0] * v[0] + A[2][1] * v[1] + A[2][2] * v[2]);
}

// mass matrix (with armature) and qfrc_smooth = clamped actuator force - bias
template <class T> void dynamics(World<T>& w) {
  std::memset(w.M, 0, sizeof(w.M));
  T bias[NV] = {};
  // velocities and velocity-product accelerations (qacc = 0), parents first
  V3<T> om[NBODY], al[NBODY], ao[NBODY];  // angular velocity, angular acc., acc. of the body origin
  V3<T> vo[NBODY];
  om[0] = al[0] = ao[0] = vo[0] = v3<T>(0, 0, 0);
  for (int b = 1; b < NBODY; b++) {
    if (b == 1) {
      om[1] = qrot(w.xq[1], v3(w.qvel[3], w.qvel[4], w.qvel[5]));
      vo[1] = v3(w.qvel[0], w.qvel[1], w.qvel[2]);
      al[1] = v3<T>(0, 0, 0);
      ao[1] = v3<T>(0, 0, 0);
    } else {
      int p = g1_body_parent[b], d = g1_body_dofadr[b];
      V3<T> r = w.xpos[b] - w.xpos[p];
      V3<T> wd = w.qvel[d] * w.wax[d];
      om[b] = om[p] + wd;
      vo[b] = vo[p] + cross(om[p], r);
      al[b] = al[p] + cross(om[p], wd);
      ao[b] = ao[p] + cross(al[p], r) + cross(om[p], cross(om[p], r));
    }
  }
  const V3<T> g = v3<T>(0, 0, T(G1_GRAVITY_Z));
  for (int b = 1; b < NBODY; b++) {
    T m = T(g1_body_mass[b]), I[3][3];
    body_inertia_world(w, b, I);
    V3<T> c = w.xipos[b] - w.xpos[b];
    V3<T> ac = ao[b] + cross(al[b], c) + cross(om[b], cross(om[b], c));
    V3<T> F = m * (ac - g);
    V3<T> N = mat3v(I, al[b]) + cross(om[b], mat3v(I, om[b]));
    V3<T> jc[NV], jr[NV];
    int ids[NV], n = 0;
    for (int i = 0; i < NV; i++)
      if (is_ancestor_dof<T>(i, b)) {
        ids[n] = i;
        jc[n] = jac_point(w, i, w.xipos[b]);
        jr[n] = w.trans[i] ? v3<T>(0, 0, 0) : w.wax[i];
        n++;
      }
    for (int a = 0; a < n; a++) {
      bias[ids[a]] += dot(jc[a], F) + dot(jr[a], N);
      V3<T> Ir = mat3v(I, jr[a]);
      for (int e = 0; e < n; e++) w.M[ids[a]][ids[e]] += m * dot(jc[a], jc[e]) + dot(jr[e], Ir);
    }
  }
  for (int i = 0; i < NV; i++) w.M[i][i] += T(g1_dof_armature[i]);
  for (int i = 0; i < NV; i++) {
    T act = 0;
    if (i >= 6) {
      const T f = T(g1_dof_kp[i]) * (w.ctrl[i - 6] - w.qpos[i + 1]) - T(g1_dof_kv[i]) * w.qvel[i];
      const T lim = T(g1_dof_frclim[i]);
      act = std::min(std::max(f, -lim), lim);
      if (w.mode) {
        ModeBase& b = w.mode->base[w.mode->k];
        const unsigned long long bit = 1ull << i;
        if (w.mode->record) {
          b.v[i] = double(w.qvel[i]);
          b.f[i] = double(f);
          if (act <= -lim || act >= lim) b.clamp |= bit;
        } else if (b.clamp & bit) {  // the base's clamp holds
          const T bound = b.f[i] > 0 ? lim : -lim;
          if (w.mode->clamp_kv == 0) {
            act = bound - T(g1_dof_kv[i]) * (w.qvel[i] - T(b.v[i]));
          } else if (w.mode->clamp_kv == 2) {
            const double o = std::max((std::fabs(b.f[i]) - double(lim)) / double(lim), 0.0);
            const T wt = w.mode->soft > 0 ? T(std::exp(-o / w.mode->soft)) : T(0);
            act = bound + wt * (f - T(b.f[i]));
          } else {
            act = bound;
          }
        } else {
          act = f;  // the base's unclamped zone holds
        }
      }
    }
    w.qfrc_smooth[i] = act - bias[i];
  }
}

// dense Cholesky A = L L' (lower triangle of L); returns false when a pivot is not positive
template <class T> bool cholesky(const T A[NV][NV], T L[NV][NV]) {
  for (int j = 0; j < NV; j++) {
    T s = A[j][j];
    for (int k = 0; k < j; k++) s -= L[j][k] * L[j][k];
    if (!(s > 0)) return false;
    L[j][j] = std::sqrt(s);
    for (int i = j + 1; i < NV; i++) {
      T t = A[i][j];
      for (int k = 0; k < j; k++) t -= L[i][k] * L[j][k];
      L[i][j] = t / L[j][j];
    }
  }
  return true;
}
template <class T> void chol_solve(const T L[NV][NV], const T* b, T* x) {
  T y[NV];
  for (int i = 0; i < NV; i++) {
    T s = b[i];
    for (int k = 0; k < i; k++) s -= L[i][k] * y[k];
    y[i] = s / L[i][i];
  }
  for (int i = NV - 1; i >= 0; i--) {
    T s = y[i];
    for (int k = i + 1; k < NV; k++) s -= L[k][i] * x[k];
    x[i] = s / L[i][i];
  }
}

// ---- collision (MuJoCo Warp's primitives as the reference uses them, margin 0) ----
template <class T> void make_frame(const V3<T>& n, V3<T> fr[3]) {
  V3<T> b = v3<T>(0, 0, 0);
  if (n[1] > T(-0.5) && n[1] < T(0.5)) b[1] = 1; else b[2] = 1;
  b = b - dot(n, b) * n;
  T bn = std::sqrt(dot(b, b));
  if (bn > 0) b = (T(1) / bn) * b;
  fr[0] = n; fr[1] = b; fr[2] = cross(n, b);
}

template <class T> V3<T> zaxis(const Q4<T>& q) { return qrot(q, v3<T>(0, 0, 1)); }

template <class T> struct GeomPose { V3<T> p; Q4<T> q; };

template <class T> void push(std::vector<Contact<T>>& out, int pair, int slot, T dist, const V3<T>& pos,
                             const V3<T> fr[3]) {
  Contact<T> c;
  c.pair = pair; c.slot = slot; c.dist = dist; c.pos = pos;
  c.frame[0] = fr[0]; c.frame[1] = fr[1]; c.frame[2] = fr[2];
  out.push_back(c);
}

// sphere core: centres p1, p2 with radii r1, r2
template <class T> void sphere_sphere(const V3<T>& p1, T r1, const V3<T>& p2, T r2, T* dist, V3<T>* pos, V3<T>* n) {
  V3<T> dir = p2 - p1;
  T d = std::sqrt(dot(dir, dir));
  *n = d == 0 ? v3<T>(1, 0, 0) : (T(1) / d) * dir;
  *dist = d - (r1 + r2);
  *pos = p1 + (r1 + T(0.5) * *dist) * *n;
}

// A contact of the sphere core between the centres c1 = p1 + x1 a1 (radius r1) and c2 = p2 + x2 a2 (r2) of pair /
// slot, pushed when dist < 0; returns dist. With a gradient mode (Mode, above): the base pass records the contact,
// the surrogate pass holds what the mode holds. hold_ok: both segment parameters free on near-parallel axes.
template <class T> T core_contact(std::vector<Contact<T>>& out, Mode* mode, int pair, int slot, const V3<T>& p1,
                                  const V3<T>& a1, T x1, T r1, const V3<T>& p2, const V3<T>& a2, T x2, T r2,
                                  bool hold_ok) {
  const ModeContact* bc = nullptr;
  if (mode && !mode->record)
    for (const ModeContact& c : mode->base[mode->k].con)
      if (c.pair == pair && c.slot == slot) { bc = &c; break; }
  if (bc && bc->hold) { x1 = T(bc->x1); x2 = T(bc->x2); }
  const V3<T> c1 = p1 + x1 * a1, c2 = p2 + x2 * a2;
  T dist; V3<T> pos, n, fr[3];
  sphere_sphere(c1, r1, c2, r2, &dist, &pos, &n);
  if (bc && mode->normal != 0) {
    const double nu = bc->nu;
    const T sc = mode->normal == 1 ? T(0) : (mode->normal == 2 ? T(nu / std::max(nu, 1e-3)) : T(nu < 1e-3 ? 0 : 1));
    const V3<T> n0 = v3(T(bc->n[0]), T(bc->n[1]), T(bc->n[2]));
    n = n0 + sc * (n - n0);
    pos = c1 + (r1 + T(0.5) * dist) * n;
  }
  make_frame(n, fr);
  if (dist < 0) {
    push(out, pair, slot, dist, pos, fr);
    if (mode && mode->record) {
      const V3<T> d = c2 - c1;
      mode->base[mode->k].con.push_back(ModeContact{pair, slot, {double(n[0]), double(n[1]), double(n[2])},
                                                    double(std::sqrt(dot(d, d))), double(x1), double(x2),
                                                    mode->normal != 0 && hold_ok});
    }
  }
  return dist;
}

template <class T> void collide(int pair, const GeomPose<T>* gp, std::vector<Contact<T>>& out, int* unsup,
                                Mode* mode) {
  int g1 = g1_pair_g1[pair], g2 = g1_pair_g2[pair], t1 = g1_geom_type[g1], t2 = g1_geom_type[g2];
  const V3<T> p1 = gp[g1].p, p2 = gp[g2].p;
  const double* s1 = g1_geom_size + 3 * g1;
  const double* s2 = g1_geom_size + 3 * g2;
  const int PLANE = 0, SPHERE = 2, CAPSULE = 3;
  if (t1 == PLANE) {
    V3<T> n = zaxis(gp[g1].q);
    if (dot(p2 - p1, n) > T(g1_geom_rbound[g2])) return;
    if (t2 == SPHERE) {
      T r = T(s2[0]);
      T dist = dot(p2, n) - dot(p1, n) - r;
      V3<T> pos = p2 - (r + T(0.5) * dist) * n, fr[3];
      make_frame(n, fr);
      if (dist < 0) push(out, pair, 0, dist, pos, fr);
    } else if (t2 == CAPSULE) {
      T r = T(s2[0]), hl = T(s2[1]);
      V3<T> ax = zaxis(gp[g2].q), fr[3];
      V3<T> b = ax - dot(n, ax) * n;  // frame tangent along the capsule axis projected on the plane
      T bn = std::sqrt(dot(b, b));
      if (bn > 0) b = (T(1) / bn) * b;
      if (bn < T(0.5)) { make_frame(n, fr); } else { fr[0] = n; fr[1] = b; fr[2] = cross(n, b); }
      for (int e = 0; e < 2; e++) {
        V3<T> ce = e == 0 ? p2 + hl * ax : p2 - hl * ax;
        T dist = dot(ce, n) - dot(p1, n) - r;
        V3<T> pos = ce - (r + T(0.5) * dist) * n;
        if (dist < 0) push(out, pair, e, dist, pos, fr);
      }
    } else {
      *unsup |= 1;
    }
    return;
  }
  V3<T> dif = p2 - p1;
  T rb = T(g1_geom_rbound[g1]) + T(g1_geom_rbound[g2]);
  if (dot(dif, dif) > rb * rb) return;  // bounding spheres apart: no contact at zero margin
  const V3<T> zero = v3<T>(0, 0, 0);
  if (t1 == SPHERE && t2 == SPHERE) {
    core_contact(out, mode, pair, 0, p1, zero, T(0), T(s1[0]), p2, zero, T(0), T(s2[0]), false);
    return;
  }
  if (t1 == SPHERE && t2 == CAPSULE) {  // closest point of the segment, MuJoCo Warp's regularised parameter
    V3<T> ax = zaxis(gp[g2].q);
    T hl = T(s2[1]);
    V3<T> a = p2 - hl * ax, ab = (T(2) * hl) * ax, ap = p1 - a;
    T gam = dot(ab, ab) + T(1e-6);
    T t = std::min(std::max(dot(ap, ab) / gam, T(0)), T(1));
    core_contact(out, mode, pair, 0, p1, zero, T(0), T(s1[0]), a, ab, t, T(s2[0]), false);
    return;
  }
  if (t1 == CAPSULE && t2 == CAPSULE) {
    V3<T> a1 = T(s1[1]) * zaxis(gp[g1].q), a2 = T(s2[1]) * zaxis(gp[g2].q), d = p1 - p2;
    T ma = dot(a1, a1), mb = -dot(a1, a2), mc = dot(a2, a2), u = -dot(a1, d), v = dot(a2, d);
    T det = ma * mc - mb * mb;
    if (std::fabs(det) >= T(1e-15)) {  // else parallel: the segments' end candidates
      T x1 = (mc * u - mb * v) / det, x2 = (ma * v - mb * u) / det;
      bool free1 = true, free2 = true;  // not set by a clamp of the cascade
      if (x1 > 1) { x1 = 1; free1 = false; x2 = (v - mb) / mc; }
      else if (x1 < -1) { x1 = -1; free1 = false; x2 = (v + mb) / mc; }
      if (x2 > 1 || x2 < -1) {
        bool hi = x2 > 1;
        x2 = hi ? T(1) : T(-1);
        free2 = false;
        T raw = hi ? (u - mb) / ma : (u + mb) / ma;
        free1 = raw > -1 && raw < 1;
        x1 = std::min(std::max(raw, T(-1)), T(1));
      }
      core_contact(out, mode, pair, 0, p1, a1, x1, T(s1[0]), p2, a2, x2, T(s2[0]),
                   free1 && free2 && det < T(1.2e-3) * ma * mc);
    } else {
      int cnt = 0;
      for (int e = 0; e < 4 && cnt < 2; e++) {
        T x1, x2;
        if (e < 2) {
          x1 = e == 0 ? T(1) : T(-1);
          T raw = e == 0 ? (v - mb) / mc : (v + mb) / mc;
          x2 = std::min(std::max(raw, T(-1)), T(1));
        } else {
          x2 = e == 2 ? T(1) : T(-1);
          T raw = e == 2 ? (u - mb) / ma : (u + mb) / ma;
          x1 = std::min(std::max(raw, T(-1)), T(1));
        }
        if (core_contact(out, mode, pair, e, p1, a1, x1, T(s1[0]), p2, a2, x2, T(s2[0]), false) <= 0) cnt++;
      }
    }
    return;
  }
  *unsup |= 1;
}

template <class T> void collision(World<T>& w) {
  GeomPose<T> gp[NGEOM];
  for (int g = 0; g < NGEOM; g++) {
    int b = g1_geom_body[g];
    gp[g].p = w.xpos[b] + qrot(w.xq[b], mv3<T>(g1_geom_pos + 3 * g));
    gp[g].q = qmul(w.xq[b], mq4<T>(g1_geom_quat + 4 * g));
  }
  std::vector<Contact<T>> all;
  for (int p = 0; p < NPAIR; p++) collide(p, gp, all, &w.unsupported, w.mode);
  w.ncon_raw = (int)all.size();
  if (w.ncon_raw > MAXCON) { w.unsupported |= 4; all.resize(MAXCON); }
  for (auto& c : all) c.mu = g1_pair_foot[c.pair] ? w.fric : T(g1_pair_mu[c.pair]);
  w.con = all;
}

// refsafe impedance: k, b and imp at the row's position (solref / solimp: the model's defaults on every row)
template <class T> void impedance(const double* solref, const double* solimp, T pos, T h, T* k, T* b, T* imp) {
  T tc = std::max(T(solref[0]), T(2) * h), dr = T(solref[1]);
  T dmin = std::min(std::max(T(solimp[0]), T(1e-4)), T(0.9999));
  T dmax = std::min(std::max(T(solimp[1]), T(1e-4)), T(0.9999));
  T width = std::max(T(1e-15), T(solimp[2]));
  T mid = std::min(std::max(T(solimp[3]), T(1e-4)), T(0.9999));
  T power = std::max(T(1), T(solimp[4]));
  *k = T(1) / std::max(T(1e-15), dmax * dmax * tc * tc * dr * dr);
  *b = T(2) / std::max(T(1e-15), dmax * tc);
  T x = std::fabs(pos) / width;
  if (x >= 1) *imp = dmax;
  else if (x <= 0) *imp = dmin;
  else {
    T y;
    if (x <= mid) y = std::pow(x, power) / std::pow(mid, power - 1);
    else y = 1 - std::pow(1 - x, power) / std::pow(1 - mid, power - 1);
    *imp = dmin + y * (dmax - dmin);
    *imp = std::min(std::max(*imp, dmin), dmax);
  }
}

template <class T> void make_rows(World<T>& w, T h) {
  int r = 0;
  // hinge limits, dof order
  for (int i = 6; i < NV && r < NEFC; i++) {
    T q = w.qpos[i + 1];
    T dlo = q - T(g1_dof_range[2 * i]), dhi = T(g1_dof_range[2 * i + 1]) - q;
    T pos = std::min(dlo, dhi);
    if (!(pos < 0)) continue;
    T sg = dlo < dhi ? T(1) : T(-1);
    std::fill(w.J[r], w.J[r] + NV, T(0));
    w.J[r][i] = sg;
    T k, b, imp;
    impedance(g1_jnt_solref, g1_jnt_solimp, pos, h, &k, &b, &imp);
    T R = std::max(T(1e-15), T(g1_dof_invweight0[i]) * (1 - imp) / imp);
    w.D[r] = T(1) / R;
    w.aref[r] = -b * (sg * w.qvel[i]) - k * imp * pos;
    r++;
  }
  // contacts, contact order
  int need = r;
  for (auto& c : w.con) need += g1_pair_dim[c.pair] == 3 ? 4 : 1;
  if (need > NEFC) w.unsupported |= 16;
  for (auto& c : w.con) {
    int dim = g1_pair_dim[c.pair];
    int b1 = g1_geom_body[g1_pair_g1[c.pair]], b2 = g1_geom_body[g1_pair_g2[c.pair]];
    T Jf[3][NV];
    for (int i = 0; i < NV; i++) {
      V3<T> jp = v3<T>(0, 0, 0);
      bool in1 = b1 > 0 && is_ancestor_dof<T>(i, b1), in2 = b2 > 0 && is_ancestor_dof<T>(i, b2);
      if (in1 != in2) {
        jp = jac_point(w, i, c.pos);
        if (in1) jp = T(-1) * jp;
      }
      for (int d = 0; d < 3; d++) Jf[d][i] = dot(c.frame[d], jp);
    }
    T vel[3];
    for (int d = 0; d < 3; d++) {
      vel[d] = 0;
      for (int i = 0; i < NV; i++) vel[d] += Jf[d][i] * w.qvel[i];
    }
    T iw = T(g1_body_invweight0[b1]) + T(g1_body_invweight0[b2]);
    if (dim == 3) iw = (c.mu * c.mu * iw + iw) * T(2) * c.mu * c.mu / T(G1_IMPRATIO);
    T k, b, imp;
    impedance(g1_pair_solref, g1_pair_solimp, c.dist, h, &k, &b, &imp);
    T R = std::max(T(1e-15), iw * (1 - imp) / imp);
    int nr = dim == 3 ? 4 : 1;
    for (int t = 0; t < nr && r < NEFC; t++, r++) {
      T sg = (t & 1) ? T(-1) : T(1);
      int tdir = 1 + (t >> 1);
      for (int i = 0; i < NV; i++) w.J[r][i] = dim == 3 ? Jf[0][i] + sg * c.mu * Jf[tdir][i] : Jf[0][i];
      T v = dim == 3 ? vel[0] + sg * c.mu * vel[tdir] : vel[0];
      w.D[r] = T(1) / R;
      w.aref[r] = -b * v - k * imp * c.dist;
    }
  }
  w.nrow = r;
}

// the Newton solver (primal, pyramidal rows are one-sided quadratics)
template <class T> struct Solver {
  World<T>& w;
  T Ma[NV], jar[NEFC];
  explicit Solver(World<T>& w_) : w(w_) {}
  void refresh(const T* a) {
    for (int i = 0; i < NV; i++) {
      T s = 0;
      for (int j = 0; j < NV; j++) s += w.M[i][j] * a[j];
      Ma[i] = s;
    }
    for (int r = 0; r < w.nrow; r++) {
      T s = 0;
      for (int i = 0; i < NV; i++) s += w.J[r][i] * a[i];
      jar[r] = s - w.aref[r];
    }
  }
  T cost(const T* a) const {
    T g = 0;
    for (int i = 0; i < NV; i++) g += T(0.5) * (Ma[i] - w.qfrc_smooth[i]) * (a[i] - w.qacc_smooth[i]);
    for (int r = 0; r < w.nrow; r++)
      if (jar[r] < 0) g += T(0.5) * w.D[r] * jar[r] * jar[r];
    return g;
  }
  void grad(T* g) const {  // M a - qfrc_smooth - J' f, f = -D jar on the active rows
    for (int i = 0; i < NV; i++) g[i] = Ma[i] - w.qfrc_smooth[i];
    for (int r = 0; r < w.nrow; r++)
      if (jar[r] < 0)
        for (int i = 0; i < NV; i++) g[i] += w.J[r][i] * w.D[r] * jar[r];
  }
  // returns the iterations run; conv: the stopping test passed
  int ls_steps = 0;  // line-search evaluations (the FLOP counter's l)
  int solve(int iterations, T tol, bool* conv) {
    T* a = w.qacc;
    const T scale = T(1) / (T(G1_MEANINERTIA) * NV);
    // warm start or qacc_smooth, whichever costs less
    refresh(a);
    T c_warm = cost(a);
    T Ma_w[NV], jar_w[NEFC], a_w[NV];
    std::copy(Ma, Ma + NV, Ma_w);
    std::copy(jar, jar + NEFC, jar_w);
    std::copy(a, a + NV, a_w);
    std::copy(w.qacc_smooth, w.qacc_smooth + NV, a);
    refresh(a);
    T c = cost(a);
    if (c > c_warm) {
      std::copy(a_w, a_w + NV, a);
      std::copy(Ma_w, Ma_w + NV, Ma);
      std::copy(jar_w, jar_w + NEFC, jar);
      c = c_warm;
    }
    T g[NV];
    grad(g);
    int it = 0;
    *conv = false;
    while (it < iterations) {
      T H[NV][NV], L[NV][NV], p[NV];
      for (int i = 0; i < NV; i++)
        for (int j = 0; j < NV; j++) H[i][j] = w.M[i][j];
      for (int r = 0; r < w.nrow; r++)
        if (jar[r] < 0)
          for (int i = 0; i < NV; i++) {
            if (w.J[r][i] == 0) continue;
            T di = w.D[r] * w.J[r][i];
            for (int j = 0; j < NV; j++) H[i][j] += di * w.J[r][j];
          }
      if (!cholesky(H, L)) break;
      T mg[NV];
      for (int i = 0; i < NV; i++) mg[i] = -g[i];
      chol_solve(L, mg, p);
      // exact line search on the piecewise quadratic along p (safeguarded 1-D Newton)
      T Mp[NV], jv[NEFC];
      for (int i = 0; i < NV; i++) {
        T s = 0;
        for (int j = 0; j < NV; j++) s += w.M[i][j] * p[j];
        Mp[i] = s;
      }
      for (int r = 0; r < w.nrow; r++) {
        T s = 0;
        for (int i = 0; i < NV; i++) s += w.J[r][i] * p[i];
        jv[r] = s;
      }
      T a1 = 0, a2 = 0;
      for (int i = 0; i < NV; i++) { a1 += (Ma[i] - w.qfrc_smooth[i]) * p[i]; a2 += p[i] * Mp[i]; }
      T alpha = 0, lo = 0, hi = T(1e30), d0 = 0;
      std::vector<char> zprev(w.nrow, 0), z(w.nrow, 0);
      bool newton = false;
      for (int k = 0; k <= 40; k++) {
        T fd = 0, fdd = 0;
        for (int r = 0; r < w.nrow; r++) {
          T x = jar[r] + alpha * jv[r];
          z[r] = x < 0;
          if (z[r]) { fd += w.D[r] * x * jv[r]; fdd += w.D[r] * jv[r] * jv[r]; }
        }
        if (newton && z == zprev) break;  // the last Newton step kept every row on its piece: exact minimiser
        if (k == 40) break;
        ls_steps++;
        fd += a1 + alpha * a2;
        fdd += a2;
        if (k == 0) { d0 = fd; if (d0 >= 0) break; }
        if (std::fabs(fd) <= T(1e-7) * std::fabs(d0)) break;
        if (fd < 0) lo = alpha; else hi = alpha;
        T nx = alpha - fd / fdd;
        newton = nx > lo && nx < hi;
        if (!newton) nx = hi < T(1e29) ? T(0.5) * (lo + hi) : T(2) * std::max(alpha, T(1e-6));
        zprev = z;
        alpha = nx;
      }
      for (int i = 0; i < NV; i++) { a[i] += alpha * p[i]; Ma[i] += alpha * Mp[i]; }
      for (int r = 0; r < w.nrow; r++) jar[r] += alpha * jv[r];
      T cnew = cost(a);
      grad(g);
      T gn = 0;
      for (int i = 0; i < NV; i++) gn += g[i] * g[i];
      gn = std::sqrt(gn);
      T improvement = scale * (c - cnew);
      c = cnew;
      it++;
      if (improvement < tol || scale * gn < tol) { *conv = true; break; }
    }
    return it;
  }
};

template <class T> int substep(World<T>& w, int iterations, T tol, int* stats) {
  const T h = T(G1_TIMESTEP);
  kinematics(w);
  dynamics(w);
  T L[NV][NV];
  if (!cholesky(w.M, L)) w.unsupported |= 64;
  chol_solve(L, w.qfrc_smooth, w.qacc_smooth);
  collision(w);
  make_rows(w, h);
  Solver<T> sv(w);
  bool conv;
  int it = sv.solve(iterations, tol, &conv);
  if (stats) { stats[0] = (int)w.con.size(); stats[1] = w.nrow; stats[2] = it; stats[3] = sv.ls_steps; }
  // implicitfast: (M + h kv) a_adv = M a*
  T A[NV][NV], rhs[NV], adv[NV];
  for (int i = 0; i < NV; i++) {
    for (int j = 0; j < NV; j++) A[i][j] = w.M[i][j];
    A[i][i] += h * T(g1_dof_kv[i]);
    rhs[i] = sv.Ma[i];
  }
  cholesky(A, L);
  chol_solve(L, rhs, adv);
  for (int i = 0; i < NV; i++) w.qvel[i] += h * adv[i];
  for (int k = 0; k < 3; k++) w.qpos[k] += h * w.qvel[k];
  {
    V3<T> om = v3(w.qvel[3], w.qvel[4], w.qvel[5]);
    T nw = std::sqrt(dot(om, om));
    if (nw > 0) {
      T ang = h * nw, sa = std::sin(ang / 2), ca = std::cos(ang / 2);
      Q4<T> dq{ca, sa * om[0] / nw, sa * om[1] / nw, sa * om[2] / nw};
      Q4<T> q{w.qpos[3], w.qpos[4], w.qpos[5], w.qpos[6]};
      Q4<T> o = qmul(q, dq);
      T on = std::sqrt(o.w * o.w + o.x * o.x + o.y * o.y + o.z * o.z);
      w.qpos[3] = o.w / on; w.qpos[4] = o.x / on; w.qpos[5] = o.y / on; w.qpos[6] = o.z / on;
    }
  }
  for (int i = 6; i < NV; i++) w.qpos[i + 1] += h * w.qvel[i];
  return it;
}

template <class T>
void step_world(int iw, const double* qpos, const double* qvel, const double* warm, const double* ctrl,
                const double* fric, const double* com, int iterations, int nsub, double tol, double* oq, double* ov,
                double* ow, int* info, int* stats, double* ocon) {
  World<T>* w = new World<T>();
  T c[NU];
  for (int i = 0; i < NQ; i++) w->qpos[i] = T(qpos[(size_t)iw * NQ + i]);
  for (int i = 0; i < NV; i++) { w->qvel[i] = T(qvel[(size_t)iw * NV + i]); w->qacc[i] = T(warm[(size_t)iw * NV + i]); }
  for (int i = 0; i < NU; i++) c[i] = T(ctrl[(size_t)iw * NU + i]);
  w->ctrl = c;
  w->fric = T(fric[iw]);
  w->com = v3(T(com[3 * iw]), T(com[3 * iw + 1]), T(com[3 * iw + 2]));
  w->unsupported = 0;
  int it = 0;
  for (int k = 0; k < nsub; k++) it = substep(*w, iterations, T(tol), stats ? stats + ((size_t)iw * nsub + k) * 4 : nullptr);
  for (int i = 0; i < NQ; i++) oq[(size_t)iw * NQ + i] = double(w->qpos[i]);
  for (int i = 0; i < NV; i++) { ov[(size_t)iw * NV + i] = double(w->qvel[i]); ow[(size_t)iw * NV + i] = double(w->qacc[i]); }
  info[4 * iw] = it;
  info[4 * iw + 1] = w->ncon_raw;
  info[4 * iw + 2] = w->nrow;
  info[4 * iw + 3] = w->unsupported;
  if (ocon)  // the last substep's kept contacts as (pair, slot, dist), pair -1 past the count
    for (int c = 0; c < MAXCON; c++) {
      double* o = ocon + ((size_t)iw * MAXCON + c) * 3;
      const bool v = c < (int)w->con.size();
      o[0] = v ? w->con[c].pair : -1.0;
      o[1] = v ? w->con[c].slot : 0.0;
      o[2] = v ? double(w->con[c].dist) : 0.0;
    }
  delete w;
}

// One world's control step from float64 inputs (qpos 36, qvel 35, warm 35, ctrl 29, fric, com 3) under a gradient
// mode's base pass or surrogate: (qpos', qvel') into out (71)
template <class T>
void mode_step(const double* q, const double* v, const double* warm, const double* u, double fric, const double* com,
               int iterations, int nsub, double tol, Mode* mode, double* out) {
  World<T>* w = new World<T>();
  T c[NU];
  for (int i = 0; i < NQ; i++) w->qpos[i] = T(q[i]);
  for (int i = 0; i < NV; i++) { w->qvel[i] = T(v[i]); w->qacc[i] = T(warm[i]); }
  for (int i = 0; i < NU; i++) c[i] = T(u[i]);
  w->ctrl = c;
  w->fric = T(fric);
  w->com = v3(T(com[0]), T(com[1]), T(com[2]));
  w->unsupported = 0;
  w->mode = mode;
  for (int k = 0; k < nsub; k++) {
    mode->k = k;
    substep(*w, iterations, T(tol), nullptr);
  }
  for (int i = 0; i < NQ; i++) out[i] = double(w->qpos[i]);
  for (int i = 0; i < NV; i++) out[NQ + i] = double(w->qvel[i]);
  delete w;
}

// qpos moved along the tangent dq (35): root position, root rotation vector in the local frame, hinge angles
void integrate_qpos(const double* q, const double* dq, double* out) {
  for (int i = 0; i < NQ; i++) out[i] = q[i];
  for (int k = 0; k < 3; k++) out[k] += dq[k];
  const double ang = std::sqrt(dq[3] * dq[3] + dq[4] * dq[4] + dq[5] * dq[5]);
  double qn = std::sqrt(q[3] * q[3] + q[4] * q[4] + q[5] * q[5] + q[6] * q[6]);
  Q4<double> quat{q[3] / qn, q[4] / qn, q[5] / qn, q[6] / qn}, dquat{1, 0, 0, 0};
  if (ang > 0) {
    const double sn = std::sin(ang / 2) / ang;
    dquat = Q4<double>{std::cos(ang / 2), sn * dq[3], sn * dq[4], sn * dq[5]};
  }
  const Q4<double> o = qmul(quat, dquat);
  out[3] = o.w; out[4] = o.x; out[5] = o.y; out[6] = o.z;
  for (int i = 6; i < NV; i++) out[i + 1] += dq[i];
}

}  // namespace

extern "C" {

// Central differences (step h) of a gradient mode's surrogate step (Mode, above: clamp_kv 0..2 with soft, normal
// 0..3), float64: J (nw, 71, 99) = d(qpos' in qpos form 36, qvel' 35) / d(qpos tangent 35, qvel 35, ctrl 29) at the
// inputs, the base pass (which records what the mode holds) run once per world. Test infrastructure: the check of the
// analytic adjoint's modes.
int g1_oracle_fd_jacobian_mode(int nw, const double* qpos, const double* qvel, const double* warm, const double* ctrl,
                               const double* fric, const double* com, int iterations, int nsub, double tol,
                               int clamp_kv, int normal, double soft, double h, int nthreads, double* J) {
  if (nw < 0 || nsub < 1 || nsub > 32 || iterations < 0 || clamp_kv < 0 || clamp_kv > 2 || normal < 0 || normal > 3)
    return 1;
  constexpr int NO = NQ + NV, NI = 2 * NV + NU;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : omp_get_max_threads())
  for (int iw = 0; iw < nw; iw++) {
    const double *q = qpos + (size_t)iw * NQ, *v = qvel + (size_t)iw * NV, *wm = warm + (size_t)iw * NV;
    const double *u = ctrl + (size_t)iw * NU, *cm = com + 3 * (size_t)iw;
    std::vector<ModeBase> base(nsub);
    Mode mode;
    mode.clamp_kv = clamp_kv; mode.normal = normal; mode.soft = soft; mode.base = base.data();
    double out[NO], plus[NO], minus[NO], qq[NQ], vv[NV], uu[NU], dq[NV];
    mode.record = true;
    mode_step<double>(q, v, wm, u, fric[iw], cm, iterations, nsub, tol, &mode, out);
    mode.record = false;
    for (int j = 0; j < NI; j++) {
      for (int sgn = 0; sgn < 2; sgn++) {
        const double d = sgn ? -h : h;
        for (int i = 0; i < NQ; i++) qq[i] = q[i];
        for (int i = 0; i < NV; i++) vv[i] = v[i];
        for (int i = 0; i < NU; i++) uu[i] = u[i];
        if (j < NV) {
          for (int i = 0; i < NV; i++) dq[i] = i == j ? d : 0.0;
          integrate_qpos(q, dq, qq);
        } else if (j < 2 * NV) {
          vv[j - NV] += d;
        } else {
          uu[j - 2 * NV] += d;
        }
        mode_step<double>(qq, vv, wm, uu, fric[iw], cm, iterations, nsub, tol, &mode, sgn ? minus : plus);
      }
      for (int o = 0; o < NO; o++) J[((size_t)iw * NO + o) * NI + j] = (plus[o] - minus[o]) / (2 * h);
    }
  }
  return 0;
}

// The base trajectory's smallest sphere-core centre distance nu over all substeps' contacts, per world (1e300 when
// it has none) with that contact's pair (-1: none), and how many capsule contacts the near-parallel rule holds:
// which states exercise the normal options. Test infrastructure.
int g1_oracle_core_stats(int nw, const double* qpos, const double* qvel, const double* warm, const double* ctrl,
                         const double* fric, const double* com, int iterations, int nsub, double* min_nu,
                         int* nholds, int* min_pair) {
  if (nw < 0 || nsub < 1 || nsub > 32) return 1;
#pragma omp parallel for schedule(dynamic, 4)
  for (int iw = 0; iw < nw; iw++) {
    std::vector<ModeBase> base(nsub);
    Mode mode;
    mode.normal = 3; mode.base = base.data(); mode.record = true;
    double out[NQ + NV];
    mode_step<double>(qpos + (size_t)iw * NQ, qvel + (size_t)iw * NV, warm + (size_t)iw * NV, ctrl + (size_t)iw * NU,
                      fric[iw], com + 3 * (size_t)iw, iterations, nsub, 1e-8, &mode, out);
    double m = 1e300;
    int nh = 0, mp = -1;
    for (const ModeBase& b : base)
      for (const ModeContact& c : b.con) {
        if (c.nu < m) { m = c.nu; mp = c.pair; }
        nh += c.hold;
      }
    min_nu[iw] = m;
    nholds[iw] = nh;
    if (min_pair) min_pair[iw] = mp;
  }
  return 0;
}

// One control step of nw worlds (row-major float64 arrays, as the C-ABI's float32 ones): nsub substeps of the
// reference's algorithm, Newton capped at `iterations` with tolerance `tol` (the model's 1e-8 by default).
// precision: 64 float64 arithmetic, 32 float32. nthreads: OpenMP threads (0: all).
// stats: NULL or (nw, nsub, 4) int32 per substep: contacts kept, constraint rows, Newton iterations, line-search
// evaluations (the inputs of the FLOP count of a step); ocon: NULL or (nw, 64, 3) float64, the last substep's kept
// contacts as (pair, slot, dist) in contact order, pair -1 past the count
int g1_oracle_step(int nw, const double* qpos, const double* qvel, const double* warm, const double* ctrl,
                   const double* fric, const double* com, int iterations, int nsub, double tol, int precision,
                   int nthreads, double* oq, double* ov, double* ow, int* info, int* stats, double* ocon) {
  if (nw < 0 || nsub < 1 || nsub > 32 || iterations < 0) return 1;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : omp_get_max_threads())
  for (int w = 0; w < nw; w++) {
    if (precision == 32)
      step_world<float>(w, qpos, qvel, warm, ctrl, fric, com, iterations, nsub, tol, oq, ov, ow, info, stats, ocon);
    else
      step_world<double>(w, qpos, qvel, warm, ctrl, fric, com, iterations, nsub, tol, oq, ov, ow, info, stats, ocon);
  }
  return 0;
}

// One substep's matrices at a given state, float64 (test infrastructure, for checking the factors a tape records):
// M (with armature), Q = M + h kv and the Newton Hessian H = M + sum D_r J_r' J_r over the rows active at qacc
// (J_r qacc - aref_r < 0), each (nw, NV, NV); nrow (nw,) the rows built. The state is the substep's input (qpos,
// qvel, ctrl, fric, com); qacc its Newton solution (reference step.py:1523 hessian at the final zones;
// host.py / step.py:1969 implicitfast for Q).
int g1_oracle_matrices(int nw, const double* qpos, const double* qvel, const double* qacc, const double* ctrl,
                       const double* fric, const double* com, double* M, double* Q, double* H, int* nrow) {
  if (nw < 0) return 1;
#pragma omp parallel for schedule(dynamic, 4)
  for (int iw = 0; iw < nw; iw++) {
    World<double>* w = new World<double>();
    double c[NU];
    for (int i = 0; i < NQ; i++) w->qpos[i] = qpos[(size_t)iw * NQ + i];
    for (int i = 0; i < NV; i++) { w->qvel[i] = qvel[(size_t)iw * NV + i]; w->qacc[i] = qacc[(size_t)iw * NV + i]; }
    for (int i = 0; i < NU; i++) c[i] = ctrl[(size_t)iw * NU + i];
    w->ctrl = c;
    w->fric = fric[iw];
    w->com = v3(com[3 * iw], com[3 * iw + 1], com[3 * iw + 2]);
    w->unsupported = 0;
    const double h = G1_TIMESTEP;
    kinematics(*w);
    dynamics(*w);
    collision(*w);
    make_rows(*w, h);
    double* m = M + (size_t)iw * NV * NV;
    double* q = Q + (size_t)iw * NV * NV;
    double* hh = H + (size_t)iw * NV * NV;
    for (int i = 0; i < NV; i++)
      for (int j = 0; j < NV; j++) {
        m[i * NV + j] = hh[i * NV + j] = q[i * NV + j] = w->M[i][j];
        if (i == j) q[i * NV + j] += h * g1_dof_kv[i];
      }
    for (int r = 0; r < w->nrow; r++) {
      double jar = -w->aref[r];
      for (int i = 0; i < NV; i++) jar += w->J[r][i] * w->qacc[i];
      if (jar < 0)
        for (int i = 0; i < NV; i++)
          for (int j = 0; j < NV; j++) hh[i * NV + j] += w->D[r] * w->J[r][i] * w->J[r][j];
    }
    nrow[iw] = w->nrow;
    delete w;
  }
  return 0;
}

// sizes: nq, nv, nu, nbody, ngeom, npair, maxcon, nefc
void g1_oracle_sizes(long long* out) {
  const long long s[8] = {NQ, NV, NU, NBODY, NGEOM, NPAIR, MAXCON, NEFC};
  for (int i = 0; i < 8; i++) out[i] = s[i];
}
}
