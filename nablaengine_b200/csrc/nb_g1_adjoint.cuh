// The analytic adjoint of a control step: the VJP from the forward tape, one warp per world, the substeps in
// reverse order. Reference: OamIcs/NablaEngine src/nablaengine/g1_engine/adjoint.py (phases A0-A8, :1-82) and
// adjoint_contact.py; the formulation here is this library's own:
//
// Per substep, with output cotangents (qbar' in the dof tangent: root translation, root rotation in the local frame,
// hinges; vbar'):
//  1. integrator: q' = q (+) h v' (root quaternion q' = q exp(h w' / 2)): vbar'_tot = vbar' + h J^T qbar' (J_r(h w')
//     the right Jacobian of SO(3) for the rotation), the input tangent gets qbar' (rotation: R(h w') qbar'_rot);
//  2. v' = v + h a_adv, (M + h kv) a_adv = M a*: y = (M + h kv)^-1 (h vbar'_tot) with L_Q,
//     abar* = h vbar'_tot - h kv y;
//  3. IFT at the Newton solution g(a*) = ID(q, v, a*) - act(q, v, u) - J' f = 0: lambda = H^-1 abar* with L_H;
//  4. the gradient of one scalar, psi = -lambda' ID(q, v, a*) + y' M(q) (a* - a_adv) + lambda' act + sum_r (J_r
//     lambda) f_r, with respect to q (tangent), v and u. Every pose dependence is collected as a wrench at the world
//     origin on the body that carries it (a cotangent pbar of a body point p is the force pbar at p: (p x pbar, pbar);
//     of a body direction d the moment d x dbar); the joint tangent cotangents are the dofs' motion vectors s_i
//     applied to the subtree sums of those wrenches (the virtual work of moving the subtree along s_i). ID's
//     recursion (velocities, accelerations, body wrenches) is reversed body by body in one leaf-to-root sweep, for two
//     channels: A (lambda; v, a*, gravity) and B (y; v = 0, a* - a_adv, no gravity). The rows' forces depend on J x for
//     x = lambda, a*, v: their cotangents are the wrench of a force at the contact point, deposited on the two bodies,
//     and enter through the motion vectors (sbar_i) and the velocity (vbar_i = s_i . wrench).
// Self contacts (sphere / capsule pairs) are differentiated through their free (unclamped) closest-point parameters
// (held where both capsule parameters are free on axes within ~2 degrees and normal != 0); the normal derivative
// kappa(d) (I - n n') of the centre distance d follows the reference's option `normal` (0 exact, 1 frozen,
// 2 1/max(d, 1e-3), 3 (default) frozen below 1e-3 m).
// clamp_kv: 0 keeps the actuator damping term on clamped dofs (MuJoCo Warp's adjoint, the API default), 1 drops it
// (exact), 2 the soft clamp surrogate with width clamp_soft.
#pragma once
#include "nb_g1_step.cuh"

namespace nbg1 {

enum : int { ADJ_REPLAY_MISMATCH = 1 << 13 };

// The world quantities the adjoint replays from the tape (the members of World it uses, same names): ~5.3 KB of
// shared memory per world instead of World's 22.5 KB
struct __align__(16) AWorld {
  float qpos[NQ], qvel[NV], qacc[NV], com[3], fric;
  float Q[NB][4], X[NB][3];            // body poses
  int ncon, nefc;
  int con_pair[MAXCON];
  unsigned char con_slot[MAXCON], con_row0[MAXCON], con_nrow[MAXCON], con_pad[MAXCON];
};
struct GeomPoses { float gx[NG][3], gq[NG][4]; };

// The adjoint's per-world state (k_adjoint: one cotangent per world; with AWorld 16.2 KB, 14 per SM). Its scratch
// overlaps by phase: the factor being solved with and its inverse diagonal (the solves, first), the replayed geom poses and the motions of a* and v with the contact batch (the
// replay and the contacts), and the sweep's subtree sums and parent cotangents (last); each phase writes its part
// after the previous owner of that space is done with it.
struct __align__(16) Adj {
  float lam[NV], y[NV], xa[NV], aadv[NV], vb[NV], qb[NV], ub[NU], u[NU];
  float qout[NV];                     // the tangent cotangent: the output's, then (from the integrator on) the input's
                                      // direct terms (integrator, limits, actuators), the sweep's added at the end
  float om[NB][3], alA[NB][3], aoA[NB][3], alB[NB][3], aoB[NB][3];  // replayed velocities / accelerations
  float VL[NB][6], VY[NB][6];         // body motions at the origin of lambda and y
  float dep[NB][24];                  // per body: G_lambda, G_a, G_v (wrenches at the origin), pose wrench
  float ax[NV][3];                    // dof axes (world)
  unsigned clamp_lo, clamp_hi;
  unsigned zone[NEFC / 32];           // the record's zone bits (row r quadratic: bit r & 31 of word r / 32)
  int nlim_tape, flags, normal, pad_;  // normal: the self-contact normal derivative option (0..3)
  union {
    struct alignas(16) {              // the solves: L_Q (tree-block order), then L_H, with its inverse diagonal;
      float L[NTRIP];                 // from a compact tape also M + h kv rebuilt for L_Q (adj_mass_factor); L and M
                                      // are written as float4 (tb_factor, adj_mass_factor): 16-byte aligned
      float dinv[NV + 1];
      float M[NTRIP];
      float Ic[NB][10];
    };
    struct {                          // the replay and the contacts
      float cw[32][30];               // a batch of 32 contacts' wrenches
      int cbody[32];                  // their bodies: b1 | b2 << 8
      float VA[NB][6], VV[NB][6];     // body motions at the origin of a* and v
      GeomPoses col;                  // geom poses
    };
    struct {                          // the sweep
      float sub[NB][36];              // subtree sums: W_A, W_B, G_lambda, G_a, G_v, P (6 each)
      float up[NB][18];               // to the parent: its om, alA, aoA, alB, aoB cotangents and the relative-position
                                      // force rbar (applied as -rbar at the parent's origin)
    };
  };
#ifdef NB_PROFILE
  long long prof_t;
#endif
};
static_assert(sizeof(AWorld) % 16 == 0 && offsetof(Adj, L) % 16 == 0 && offsetof(Adj, M) % 16 == 0,
              "the solves' factor and mass-matrix scratch are written as float4");

// What every cotangent of a record shares (the Jacobian's preparation: its per-record replay beside AWorld)
struct __align__(16) AdjShared {
  float xa[NV], aadv[NV], u[NU];
  GeomPoses col;                      // geom poses
  float om[NB][3], alA[NB][3], aoA[NB][3], alB[NB][3], aoB[NB][3];
  float VA[NB][6], VV[NB][6];
  float ax[NV][3];
  unsigned clamp_lo, clamp_hi;
  unsigned zone[NEFC / 32];
  int nlim_tape, pad_[3];
};

// ---- replay ---------------------------------------------------------------------------------------------------------
// poses, the dofs' axes and both channels' velocities / accelerations (lane = body, by depth level)
template <class SH>
__device__ __noinline__ void adj_replay_kin(AWorld& s, SH& W, int lane) {
  // lane = body. Poses by pointer jumping over the ancestors (a rigid transform composes associatively: 4 rounds
  // for depths up to 15), then the velocities and both channels' accelerations as path sums of per-body increments
  // (each increment needs only its parent's already-summed quantities), 4 rounds each: 16 dependent rounds
  // instead of 11 levels of the whole recursion
  static_assert(MAXD < 16, "4 pointer-jumping rounds");
  const int b = lane;
  const bool body = b >= 1 && b < NB;
  const int p = b >= 2 && b < NB ? ldi(g1_body_parent + b) : 0, d = b + 4;
  float Q[4] = {1.f, 0.f, 0.f, 0.f}, X[3] = {0.f, 0.f, 0.f}, axl[3] = {0.f, 0.f, 0.f};
  if (b == 1) {
    const float q[4] = {s.qpos[3], s.qpos[4], s.qpos[5], s.qpos[6]};
    const float n = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
    for (int k = 0; k < 4; k++) Q[k] = q[k] / n;
    for (int k = 0; k < 3; k++) X[k] = s.qpos[k];
  } else if (body) {  // the transform relative to the parent: body_pos, body_quat (x) axis-angle(hinge)
    const float bq[4] = {ld(g1_body_quat + 4 * b), ld(g1_body_quat + 4 * b + 1), ld(g1_body_quat + 4 * b + 2),
                         ld(g1_body_quat + 4 * b + 3)};
    for (int k = 0; k < 3; k++) { X[k] = ld(g1_body_pos + 3 * b + k); axl[k] = ld(g1_body_axis + 3 * b + k); }
    float sn, cs;
    sincosf(0.5f * s.qpos[d + 1], &sn, &cs);
    const float ha[4] = {cs, sn * axl[0], sn * axl[1], sn * axl[2]};
    qmul(bq, ha, Q);
  }
  int par = p;
#pragma unroll
  for (int round = 0; round < 4; round++) {
    float Qa[4], Xa[3], Qn[4], t[3];
#pragma unroll
    for (int k = 0; k < 4; k++) Qa[k] = __shfl_sync(FULL, Q[k], par);
#pragma unroll
    for (int k = 0; k < 3; k++) Xa[k] = __shfl_sync(FULL, X[k], par);
    qmul(Qa, Q, Qn);
    qrot(Qa, X, t);
    for (int k = 0; k < 4; k++) Q[k] = Qn[k];
    for (int k = 0; k < 3; k++) X[k] = Xa[k] + t[k];
    par = __shfl_sync(FULL, par, par);
  }
  // the dof axes (world), the parent's pose and this body's lever arm r = X - X_parent
  float w[3] = {0.f, 0.f, 0.f}, r[3];
  if (b >= 2 && b < NB) qrot(Q, axl, w);
  float Xp[3];
  for (int k = 0; k < 3; k++) { Xp[k] = __shfl_sync(FULL, X[k], p); r[k] = X[k] - Xp[k]; }
  const float vd = b >= 2 && b < NB ? s.qvel[d] : 0.f, ad = b >= 2 && b < NB ? s.qacc[d] : 0.f;
  const float xd = b >= 2 && b < NB ? W.xa[d] : 0.f;
  // path sums: om (increment w vd; the root R w_local)
  auto path_sum = [&](float* a) {
    int pp = p;
#pragma unroll
    for (int round = 0; round < 4; round++) {
#pragma unroll
      for (int k = 0; k < 3; k++) a[k] += __shfl_sync(FULL, a[k], pp);
      pp = __shfl_sync(FULL, pp, pp);
    }
  };
  float om[3] = {0.f, 0.f, 0.f}, alA[3] = {0.f, 0.f, 0.f}, alB[3] = {0.f, 0.f, 0.f};
  if (b == 1) {
    const float wl[3] = {s.qvel[3], s.qvel[4], s.qvel[5]};
    const float al[3] = {s.qacc[3], s.qacc[4], s.qacc[5]}, xl[3] = {W.xa[3], W.xa[4], W.xa[5]};
    qrot(Q, wl, om);
    qrot(Q, al, alA);
    qrot(Q, xl, alB);
  } else if (body) {
    for (int k = 0; k < 3; k++) om[k] = w[k] * vd;
  }
  path_sum(om);
  // angular accelerations: increments om_p x (w vd) + w ad (channel A), w xd (channel B)
  float omp[3];
  for (int k = 0; k < 3; k++) omp[k] = __shfl_sync(FULL, om[k], p);
  if (b >= 2 && b < NB) {
    const float wv[3] = {w[0] * vd, w[1] * vd, w[2] * vd};
    float u[3];
    cross(omp, wv, u);
    for (int k = 0; k < 3; k++) { alA[k] = u[k] + w[k] * ad; alB[k] = w[k] * xd; }
  }
  path_sum(alA);
  path_sum(alB);
  // origin accelerations: increments alA_p x r + om_p x (om_p x r), alB_p x r; the root's (a_lin - g, xa_lin)
  float aoA[3] = {0.f, 0.f, 0.f}, aoB[3] = {0.f, 0.f, 0.f};
  {
    float alAp[3], alBp[3];
    for (int k = 0; k < 3; k++) { alAp[k] = __shfl_sync(FULL, alA[k], p); alBp[k] = __shfl_sync(FULL, alB[k], p); }
    if (b == 1) {
      for (int k = 0; k < 3; k++) { aoA[k] = s.qacc[k]; aoB[k] = W.xa[k]; }
      aoA[2] -= G1_GRAVITY_Z;
    } else if (body) {
      float u2[3], u3[3], u4[3], u5[3];
      cross(alAp, r, u2);
      cross(omp, r, u3);
      cross(omp, u3, u4);
      cross(alBp, r, u5);
      for (int k = 0; k < 3; k++) { aoA[k] = u2[k] + u4[k]; aoB[k] = u5[k]; }
    }
  }
  path_sum(aoA);
  path_sum(aoB);
  if (b < NB) {
    for (int k = 0; k < 4; k++) s.Q[b][k] = Q[k];
    for (int k = 0; k < 3; k++) {
      s.X[b][k] = X[k];
      W.om[b][k] = om[k]; W.alA[b][k] = alA[k]; W.aoA[b][k] = aoA[k]; W.alB[b][k] = alB[k]; W.aoB[b][k] = aoB[k];
    }
    if (b >= 2)
      for (int k = 0; k < 3; k++) W.ax[d][k] = w[k];
    if (b == 1)
      for (int k = 0; k < 3; k++) {
        const float e[3] = {k == 0 ? 1.f : 0.f, k == 1 ? 1.f : 0.f, k == 2 ? 1.f : 0.f};
        float wk[3];
        qrot(Q, e, wk);
        for (int t = 0; t < 3; t++) { W.ax[3 + k][t] = wk[t]; W.ax[k][t] = e[t]; }
      }
  }
  __syncwarp();
}

// the motion of body b (angular, linear velocity of the world origin) for the generalised vector v: pointer jumping
// over the ancestor dofs, with the motion vectors s_i = (w_i, X_b x w_i) (root translations: (0, e_k))
template <class SH>
__device__ __noinline__ void adj_motion(const AWorld& s, const SH& W, const float* v, float (*out)[6],
                                      int lane) {
  float a[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int par = 0;
  if (lane == 1) {
    for (int k = 0; k < 3; k++) {
      a[k] = v[3] * W.ax[3][k] + v[4] * W.ax[4][k] + v[5] * W.ax[5][k];
      a[3 + k] = v[k];
    }
    float xw[3];
    cross(s.X[1], a, xw);  // rotations about the root origin: linear part X_1 x w
    for (int k = 0; k < 3; k++) a[3 + k] += xw[k];
  } else if (lane >= 2 && lane < NB) {
    const int d = lane + 4;
    const float vd = v[d];
    float xw[3];
    cross(s.X[lane], W.ax[d], xw);
    for (int k = 0; k < 3; k++) { a[k] = vd * W.ax[d][k]; a[3 + k] = vd * xw[k]; }
    par = ldi(g1_body_parent + lane);
  }
#pragma unroll
  for (int round = 0; round < 4; round++) {
#pragma unroll
    for (int k = 0; k < 6; k++) a[k] += __shfl_sync(FULL, a[k], par);
    par = __shfl_sync(FULL, par, par);
  }
  if (lane < NB)
    for (int k = 0; k < 6; k++) out[lane][k] = a[k];
  __syncwarp();
}

// make_frame's VJP: rows n, b = normalize(e - n (n . e)), c = n x b; frb = cotangents of the 3 rows -> nbar
__device__ __forceinline__ void make_frame_vjp(const float* n, const float* frb, float* nbar) {
  float e[3] = {0.f, 0.f, 0.f};
  if (n[1] > -0.5f && n[1] < 0.5f) e[1] = 1.f; else e[2] = 1.f;
  const float ne = dot3(n, e);
  float b0[3];
  for (int k = 0; k < 3; k++) b0[k] = e[k] - n[k] * ne;
  const float bn = sqrtf(dot3(b0, b0));
  float b[3];
  for (int k = 0; k < 3; k++) b[k] = b0[k] / bn;
  float bb[3], t[3];
  cross(frb + 6, n, t);  // c = n x b: bbar += cbar x n, nbar += b x cbar
  for (int k = 0; k < 3; k++) bb[k] = frb[3 + k] + t[k];
  cross(b, frb + 6, t);
  for (int k = 0; k < 3; k++) nbar[k] += frb[k] + t[k];
  const float bdb = dot3(b, bb);
  float b0b[3];
  for (int k = 0; k < 3; k++) b0b[k] = (bb[k] - b[k] * bdb) / bn;
  const float nb0 = dot3(n, b0b);
  for (int k = 0; k < 3; k++) nbar[k] += -ne * b0b[k] - e[k] * nb0;
}

// impedance and its derivative in the position: imp, dimp / dpos (power-2 solimp, as the forward's impedance)
__device__ __forceinline__ void impedance_d(const float* solimp, float pos, float* imp, float* dimp) {
  const float dmin = fminf(fmaxf(solimp[0], 1e-4f), 0.9999f), dmax = fminf(fmaxf(solimp[1], 1e-4f), 0.9999f);
  const float width = fmaxf(1e-15f, solimp[2]), mid = fminf(fmaxf(solimp[3], 1e-4f), 0.9999f);
  const float x = fabsf(pos) / width;
  if (x >= 1.f) { *imp = dmax; *dimp = 0.f; return; }
  if (x <= 0.f) { *imp = dmin; *dimp = 0.f; return; }
  float y, dy;
  if (x <= mid) { y = x * x / mid; dy = 2.f * x / mid; }
  else { y = 1.f - (1.f - x) * (1.f - x) / (1.f - mid); dy = 2.f * (1.f - x) / (1.f - mid); }
  const float v = dmin + y * (dmax - dmin);
  if (v < dmin || v > dmax) { *imp = fminf(fmaxf(v, dmin), dmax); *dimp = 0.f; return; }
  *imp = v;
  *dimp = (dmax - dmin) * dy * (pos < 0.f ? -1.f : 1.f) / width;
}

// ---- the rows' terms ------------------------------------------------------------------------------------------------
// One contact's terms (one thread, no warp operations): replay the tape's contact (pair, slot) from the geom poses,
// its rows' forces at the tape's zones, the cotangents of J x for x = lambda, a*, v as forces at the contact point
// (wrenches at the origin, deposited on the two bodies) and the geometry's pose wrenches. Everything but lambda's
// part is the same for every cotangent and is computed once; the terms of lambda are linear in its relative motion
// between the two bodies, dV = V^lambda(b2) - V^lambda(b1) (angular, linear at the origin), and are evaluated NEVAL
// times: dvl(e, b1, b2, dV) gives the e-th dV, put(e, out, b) takes out[30]: G(lambda), G(a*), G(v) (out[0..17], G as
// deposited on body 2: G(lambda) does not depend on dV, and G(v) is b G(a*) up to rounding, b the rows' damping),
// the pose wrenches of body 2 (out[18..23]) and body 1 (out[24..29]; zero for a plane). Returns the replay mismatch
// flag (the replayed distance is not negative).
template <int NEVAL, class SH, class DV, class PUT>
__device__ __forceinline__ int contact_terms(const AWorld& s, const SH& W, int c, int normal, DV dvl, PUT put) {
  int mismatch = 0;
  {
    const int pr = s.con_pair[c], slot = s.con_slot[c];
    const int g1 = ldi(g1_pair_g1 + pr), g2 = ldi(g1_pair_g2 + pr);
    const int t1 = ldi(g1_geom_type + g1), t2 = ldi(g1_geom_type + g2);
    const int b1 = ldi(g1_geom_body + g1), b2 = ldi(g1_geom_body + g2);
    const int dim = ldi(g1_pair_dim + pr);
    const float mu = dim != 3 ? 0.f : (ldi(g1_pair_foot + pr) ? s.fric : ld(g1_pair_mu + pr));
    float p1[3], p2[3];
    for (int k = 0; k < 3; k++) { p1[k] = W.col.gx[g1][k]; p2[k] = W.col.gx[g2][k]; }
    const float r1 = ld(g1_geom_size + 3 * g1), r2 = ld(g1_geom_size + 3 * g2);
    // geometry: the two sphere-core points (v1 on body 1, v2 on body 2), or the plane case
    float dist = 0.f, pos[3], fr[9], nrm[3], v1[3], v2[3], ax[3] = {0.f, 0.f, 0.f}, proj = 0.f;
    const bool plane = t1 == 0;
    // the segment parameters of the self contacts and whether each is free (not clamped: differentiated); sphere-
    // capsule: x2 = t on [a, a + ab] (sa = a, sb = ab, sd = ap, ma = ab . ab + 1e-6); capsule-capsule: x1, x2 on the
    // half-axes sa = a1 hl1, sb = a2 hl2 with sd = p1 - p2 and the 2 x 2 system (ma, mb, mc) x = (uu, vv)
    float sa[3] = {0.f, 0.f, 0.f}, sb[3] = {0.f, 0.f, 0.f}, sd[3] = {0.f, 0.f, 0.f}, axu[3] = {0.f, 0.f, 0.f};
    float ma = 1.f, mb = 0.f, mc = 1.f, x1 = 0.f, x2 = 0.f;
    bool fr1 = false, fr2 = false;
    if (plane) {
      zaxis(W.col.gq[g1], nrm);
      if (t2 == 3) {
        zaxis(W.col.gq[g2], ax);
        const float hl = ld(g1_geom_size + 3 * g2 + 1);
        for (int k = 0; k < 3; k++) v2[k] = slot == 0 ? p2[k] + hl * ax[k] : p2[k] - hl * ax[k];
        const float na = dot3(nrm, ax);
        float pb[3] = {ax[0] - nrm[0] * na, ax[1] - nrm[1] * na, ax[2] - nrm[2] * na};
        proj = sqrtf(dot3(pb, pb));
        if (proj < 0.5f) make_frame(nrm, fr);
        else {
          for (int k = 0; k < 3; k++) pb[k] /= proj;
          float cc[3];
          cross(nrm, pb, cc);
          for (int k = 0; k < 3; k++) { fr[k] = nrm[k]; fr[3 + k] = pb[k]; fr[6 + k] = cc[k]; }
        }
      } else {
        for (int k = 0; k < 3; k++) v2[k] = p2[k];
        make_frame(nrm, fr);
      }
      dist = dot3(v2, nrm) - dot3(p1, nrm) - r2;
      const float hp = r2 + 0.5f * dist;
      for (int k = 0; k < 3; k++) pos[k] = v2[k] - nrm[k] * hp;
    } else {
      if (t1 == 2 && t2 == 2) {
        for (int k = 0; k < 3; k++) { v1[k] = p1[k]; v2[k] = p2[k]; }
      } else if (t1 == 2 && t2 == 3) {
        const float hl = ld(g1_geom_size + 3 * g2 + 1);
        zaxis(W.col.gq[g2], axu);
        for (int k = 0; k < 3; k++) { sa[k] = p2[k] - axu[k] * hl; sb[k] = 2.f * hl * axu[k]; sd[k] = p1[k] - sa[k]; }
        ma = dot3(sb, sb) + 1e-6f;
        const float raw = dot3(sd, sb) / ma;
        fr2 = raw > 0.f && raw < 1.f;
        x2 = fminf(fmaxf(raw, 0.f), 1.f);
        for (int k = 0; k < 3; k++) { v1[k] = p1[k]; v2[k] = sa[k] + x2 * sb[k]; }
      } else {
        const float hl1 = ld(g1_geom_size + 3 * g1 + 1), hl2 = ld(g1_geom_size + 3 * g2 + 1);
        zaxis(W.col.gq[g1], sa);
        zaxis(W.col.gq[g2], sb);
        for (int k = 0; k < 3; k++) { sa[k] *= hl1; sb[k] *= hl2; sd[k] = p1[k] - p2[k]; }
        ma = dot3(sa, sa); mb = -dot3(sa, sb); mc = dot3(sb, sb);
        const float uu = -dot3(sa, sd), vv = dot3(sb, sd);
        const float det = ma * mc - mb * mb;
        if (fabsf(det) >= 1e-15f) {
          x1 = (mc * uu - mb * vv) / det; x2 = (ma * vv - mb * uu) / det;
          fr1 = fr2 = true;
          if (x1 > 1.f) { x1 = 1.f; fr1 = false; x2 = (vv - mb) / mc; }
          else if (x1 < -1.f) { x1 = -1.f; fr1 = false; x2 = (vv + mb) / mc; }
          if (x2 > 1.f || x2 < -1.f) {
            const bool hi = x2 > 1.f;
            x2 = hi ? 1.f : -1.f;
            fr2 = false;
            const float raw = hi ? (uu - mb) / ma : (uu + mb) / ma;
            fr1 = raw > -1.f && raw < 1.f;
            x1 = fminf(fmaxf(raw, -1.f), 1.f);
          }
          // both free on near-parallel axes, with a normal option: both held (sin^2 of the angle < 1.2e-3)
          if (normal != 0 && fr1 && fr2 && det < 1.2e-3f * ma * mc) fr1 = fr2 = false;
        } else if (slot < 2) {
          x1 = slot == 0 ? 1.f : -1.f;
          const float raw = slot == 0 ? (vv - mb) / mc : (vv + mb) / mc;
          fr2 = raw > -1.f && raw < 1.f;
          x2 = fminf(fmaxf(raw, -1.f), 1.f);
        } else {
          x2 = slot == 2 ? 1.f : -1.f;
          const float raw = slot == 2 ? (uu - mb) / ma : (uu + mb) / ma;
          fr1 = raw > -1.f && raw < 1.f;
          x1 = fminf(fmaxf(raw, -1.f), 1.f);
        }
        for (int k = 0; k < 3; k++) { v1[k] = p1[k] + sa[k] * x1; v2[k] = p2[k] + sb[k] * x2; }
      }
      sphere_sphere(v1, r1, v2, r2, &dist, pos, nrm);
      make_frame(nrm, fr);
    }
    mismatch = !(dist < 0.f);
    // rows: D (1 / R), the impedance and its derivative, stiffness k and damping b
    float iw = ld(g1_body_invweight0 + b1) + ld(g1_body_invweight0 + b2);
    if (dim == 3) iw = (mu * mu * iw + iw) * 2.f * mu * mu / (float)G1_IMPRATIO;
    const float h = G1_TIMESTEP;
    const float sr[2] = {ld(g1_pair_solref), ld(g1_pair_solref + 1)};
    const float si[5] = {ld(g1_pair_solimp), ld(g1_pair_solimp + 1), ld(g1_pair_solimp + 2), ld(g1_pair_solimp + 3),
                         ld(g1_pair_solimp + 4)};
    float kk, bb, imp0, imp, dimp;
    impedance(sr, si, dist, h, &kk, &bb, &imp0);
    impedance_d(si, dist, &imp, &dimp);
    const float R = fmaxf(1e-15f, iw * (1.f - imp) / imp), D = 1.f / R;
    const float dD = R > 1e-15f ? D * D * iw / (imp * imp) : 0.f;  // dD / dimp = 1 / (iw (1 - imp)^2)
    // the motions of a* (m = 1) and v (m = 2) at the contact point: u = dV_lin + dW x pos, jd_d = fr_d . u; the
    // rows' Bt = J_t a + b J_t v + k imp dist and Abar = -D Bt, the cotangent of J_t lambda, which gives G(lambda)
    float u[3][3], jd[3][3], dW[3][3];
    for (int m = 1; m < 3; m++) {
      const float(*B)[6] = m == 1 ? W.VA : W.VV;
      float dV[6], t[3];
      for (int k = 0; k < 6; k++) dV[k] = B[b2][k] - B[b1][k];
      cross(dV, pos, t);
      for (int k = 0; k < 3; k++) { u[m][k] = dV[3 + k] + t[k]; dW[m][k] = dV[k]; }
      for (int dd = 0; dd < 3; dd++) jd[m][dd] = dot3(fr + 3 * dd, u[m]);
    }
    // psi_c = -D sum_t (J_t lambda) (J_t a + b J_t v + k imp dist) over the tape's quadratic rows (at most 4)
    const int r0 = s.con_row0[c], nr = s.con_nrow[c];
    const float kterm = kk * imp * dist;
    float jdb0[3] = {0.f, 0.f, 0.f}, Bt[4] = {0.f, 0.f, 0.f, 0.f};
    unsigned quad = 0u;  // bit t: row r0 + t is quadratic
#pragma unroll
    for (int t = 0; t < 4; t++) {
      if (t >= nr) break;
      const int r = r0 + t;
      if (!((W.zone[r >> 5] >> (r & 31)) & 1u)) continue;
      quad |= 1u << t;
      const float sg = (t & 1) ? -1.f : 1.f;
      const int kd = 1 + (t >> 1);
      const float w1 = dim == 3 ? sg * mu : 0.f;
      const float Ja = jd[1][0] + w1 * jd[1][kd], Jv = jd[2][0] + w1 * jd[2][kd];
      Bt[t] = Ja + bb * Jv + kterm;
      const float Abar = -D * Bt[t];
      jdb0[0] += Abar;
      if (dim == 3) jdb0[kd] += w1 * Abar;
    }
    float out[30];
    {
      float ub0[3] = {0.f, 0.f, 0.f}, t[3];
      for (int dd = 0; dd < 3; dd++)
        for (int k = 0; k < 3; k++) ub0[k] += jdb0[dd] * fr[3 * dd + k];
      cross(pos, ub0, t);
      for (int k = 0; k < 3; k++) { out[k] = t[k]; out[3 + k] = ub0[k]; }
    }
#pragma unroll 1
    for (int e = 0; e < NEVAL; e++) {
      // lambda's terms: u(lambda) from dV; the rows' Bbar = -D J_t lambda (the cotangent of J_t a; b Bbar of J_t v),
      // the cotangents of D and of k imp dist
      {
        float dVl[6], t[3];
        dvl(e, b1, b2, dVl);
        cross(dVl, pos, t);
        for (int k = 0; k < 3; k++) { u[0][k] = dVl[3 + k] + t[k]; dW[0][k] = dVl[k]; }
        for (int dd = 0; dd < 3; dd++) jd[0][dd] = dot3(fr + 3 * dd, u[0]);
      }
      float jdb[3][3] = {{jdb0[0], jdb0[1], jdb0[2]}, {0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}};
      float Dbar = 0.f, kterm_bar = 0.f;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        if (!((quad >> t) & 1u)) continue;
        const float sg = (t & 1) ? -1.f : 1.f;
        const int kd = 1 + (t >> 1);
        const float w1 = dim == 3 ? sg * mu : 0.f;
        const float Jl = jd[0][0] + w1 * jd[0][kd];
        const float Bbar = -D * Jl;
        Dbar -= Jl * Bt[t];
        kterm_bar += Bbar;
        jdb[1][0] += Bbar;
        jdb[2][0] += bb * Bbar;
        if (dim == 3) {
          jdb[1][kd] += w1 * Bbar;
          jdb[2][kd] += w1 * (bb * Bbar);
        }
      }
      // back through jd = fr . u: ubar(x), frame cotangents, pos cotangent
      float frb[9], pb[3] = {0.f, 0.f, 0.f};
      for (int k = 0; k < 9; k++) frb[k] = 0.f;
      for (int m = 0; m < 3; m++) {
        float ub[3] = {0.f, 0.f, 0.f}, t[3];
        for (int dd = 0; dd < 3; dd++)
          for (int k = 0; k < 3; k++) { ub[k] += jdb[m][dd] * fr[3 * dd + k]; frb[3 * dd + k] += jdb[m][dd] * u[m][k]; }
        // u = dV_lin + dW x pos: the wrench (pos x ubar, ubar); pos gets ubar x dW
        cross(ub, dW[m], t);
        for (int k = 0; k < 3; k++) pb[k] += t[k];
        if (m > 0) {
          cross(pos, ub, t);
          for (int k = 0; k < 3; k++) { out[6 * m + k] = t[k]; out[6 * m + 3 + k] = ub[k]; }
        }
      }
      for (int k = 18; k < 30; k++) out[k] = 0.f;
      // dist: through imp (D, k imp dist)
      const float distb = kterm_bar * kk * (imp + dimp * dist) + Dbar * dD * dimp;
      // geometry VJP -> pose forces at v1 (body 1) and v2 (body 2) and moments
      float v1b[3] = {0.f, 0.f, 0.f}, v2b[3] = {0.f, 0.f, 0.f}, m2[3] = {0.f, 0.f, 0.f};
      if (plane) {
        // pos = v2 - n (r2 + dist / 2), dist = n . v2 - n . p1 - r2 (plane fixed: the world)
        const float np = dot3(nrm, pb);
        for (int k = 0; k < 3; k++) v2b[k] = pb[k] - 0.5f * nrm[k] * np + nrm[k] * distb;
        if (t2 == 3 && proj >= 0.5f) {  // frame along the axis projected on the plane
          float bbv[3], t[3];
          cross(frb + 6, nrm, t);
          for (int k = 0; k < 3; k++) bbv[k] = frb[3 + k] + t[k];
          const float* bvec = fr + 3;
          const float bd = dot3(bvec, bbv);
          float pjb[3];
          for (int k = 0; k < 3; k++) pjb[k] = (bbv[k] - bvec[k] * bd) / proj;
          const float npj = dot3(nrm, pjb);
          float axb[3];
          for (int k = 0; k < 3; k++) axb[k] = pjb[k] - nrm[k] * npj;
          cross(ax, axb, m2);  // a body direction: moment ax x axbar
        }
      } else {
        // pos = v1 + n (r1 + dist / 2), dist = |v2 - v1| - r1 - r2, n = (v2 - v1) / |v2 - v1|, frame = make_frame(n)
        float nb[3];
        const float hp = r1 + 0.5f * dist;
        for (int k = 0; k < 3; k++) nb[k] = hp * pb[k];
        const float distb2 = distb + 0.5f * dot3(nrm, pb);
        make_frame_vjp(nrm, frb, nb);
        float dirb[3];
        const float dd = dist + r1 + r2;
        // kappa(dd) of the normal derivative kappa (I - n n'): 0 exact 1/dd, 1 frozen frame, 2 1/max(dd, eps),
        // 3 frozen below eps (strict <), eps = 1e-3 m
        const int nopt = normal;
        const float kap =
            nopt == 1 ? 0.f : (nopt == 2 ? 1.f / fmaxf(dd, 1e-3f) : (nopt == 3 && dd < 1e-3f ? 0.f : 1.f / dd));
        const float nnb = dot3(nrm, nb);
        for (int k = 0; k < 3; k++) dirb[k] = nrm[k] * distb2 + kap * (nb[k] - nrm[k] * nnb);
        for (int k = 0; k < 3; k++) { v1b[k] = pb[k] - dirb[k]; v2b[k] = dirb[k]; }
      }
      float t[3];
      if (plane) {
        cross(v2, v2b, t);
        for (int k = 0; k < 3; k++) { out[18 + k] = t[k] + m2[k]; out[21 + k] = v2b[k]; }
      } else {
        // the core points back to the geoms: forces P1 at p1, P2 at p2 and moments m1, m2 of the axes' cotangents,
        // through the free segment parameters
        float P1[3], P2[3], m1[3] = {0.f, 0.f, 0.f};
        if (t1 == 2 && t2 == 2) {
          for (int k = 0; k < 3; k++) { P1[k] = v1b[k]; P2[k] = v2b[k]; }
        } else if (t1 == 2) {  // sphere-capsule: v2 = sa + x2 sb, x2 = (sd . sb) / ma, sd = p1 - sa
          const float hl = ld(g1_geom_size + 3 * g2 + 1);
          const float xb = fr2 ? dot3(v2b, sb) : 0.f, sdb = dot3(sd, sb);
          float sdbar[3], sbb[3], sab[3];
          for (int k = 0; k < 3; k++) {
            sdbar[k] = xb * sb[k] / ma;
            sbb[k] = x2 * v2b[k] + xb * sd[k] / ma - 2.f * xb * sdb * sb[k] / (ma * ma);
            sab[k] = v2b[k] - sdbar[k];
            P1[k] = v1b[k] + sdbar[k];
            P2[k] = sab[k];
          }
          float axb[3];
          for (int k = 0; k < 3; k++) axb[k] = -hl * sab[k] + 2.f * hl * sbb[k];
          cross(axu, axb, m2);
        } else {  // capsule-capsule: v1 = p1 + sa x1, v2 = p2 + sb x2
          const float xb1 = fr1 ? dot3(v1b, sa) : 0.f, xb2 = fr2 ? dot3(v2b, sb) : 0.f;
          float ub = 0.f, vb = 0.f, mab = 0.f, mbb = 0.f, mcb = 0.f;
          if (fr1 && fr2) {
            const float det = ma * mc - mb * mb;
            const float z1 = (mc * xb1 - mb * xb2) / det, z2 = (ma * xb2 - mb * xb1) / det;
            ub = z1; vb = z2; mab = -z1 * x1; mbb = -(z1 * x2 + z2 * x1); mcb = -z2 * x2;
          } else if (fr2) {  // x2 = (vv - mb x1) / mc
            vb = xb2 / mc; mbb = -x1 * xb2 / mc; mcb = -x2 * xb2 / mc;
          } else if (fr1) {  // x1 = (uu - mb x2) / ma
            ub = xb1 / ma; mbb = -x2 * xb1 / ma; mab = -x1 * xb1 / ma;
          }
          float sab[3], sbb[3], sdb[3];
          for (int k = 0; k < 3; k++) {
            sab[k] = x1 * v1b[k] + 2.f * mab * sa[k] - mbb * sb[k] - ub * sd[k];
            sbb[k] = x2 * v2b[k] - mbb * sa[k] + 2.f * mcb * sb[k] + vb * sd[k];
            sdb[k] = -ub * sa[k] + vb * sb[k];
            P1[k] = v1b[k] + sdb[k];
            P2[k] = v2b[k] - sdb[k];
          }
          cross(sa, sab, m1);  // the half-axes are body directions scaled by their half lengths
          cross(sb, sbb, m2);
        }
        cross(p2, P2, t);
        for (int k = 0; k < 3; k++) { out[18 + k] = t[k] + m2[k]; out[21 + k] = P2[k]; }
        cross(p1, P1, t);
        for (int k = 0; k < 3; k++) { out[24 + k] = t[k] + m1[k]; out[27 + k] = P1[k]; }
      }
      put(e, (const float*)out, bb);
    }
  }
  return mismatch;
}

// Contacts (lane = contact): one batch of 32 contacts' terms for the cotangent of A (the motion of lambda in A.VL)
// into cw, their bodies into A.cbody. Returns the replay mismatch flag of this lane.
template <class SH, class RW>
__device__ __noinline__ int adj_contacts(AWorld& s, const SH& W, RW& A, const float* rec, float (*cw)[30], int c0,
                                        int lane) {
  const int c = c0 + lane;
  float out[30];
  for (int k = 0; k < 30; k++) out[k] = 0.f;
  int mismatch = 0;
  if (c < s.ncon) {
    mismatch = contact_terms<1>(
        s, W, c, A.normal,
        [&](int, int b1, int b2, float* dV) {
          for (int k = 0; k < 6; k++) dV[k] = A.VL[b2][k] - A.VL[b1][k];
        },
        [&](int, const float* o, float) {
          for (int k = 0; k < 30; k++) out[k] = o[k];
        });
    const int pr = s.con_pair[c];
    A.cbody[lane] = ldi(g1_geom_body + ldi(g1_pair_g1 + pr)) | ldi(g1_geom_body + ldi(g1_pair_g2 + pr)) << 8;
  }
  for (int k = 0; k < 30; k++) cw[lane][k] = out[k];
  __syncwarp();
  return mismatch;
}

// lane = body: adds the batch's contact terms (contacts c0 .. c0 + 31, in contact order): G(x) with sign + on body 2,
// - on body 1; the pose wrenches of each body's points
template <class RW>
__device__ __noinline__ void adj_contact_deposit(const AWorld& s, RW& A, const float (*cw)[30], int c0, int lane) {
  const int n = min(32, s.ncon - c0);
  if (lane < NB && lane > 0) {
    float acc[24];
    for (int k = 0; k < 24; k++) acc[k] = A.dep[lane][k];
    for (int i = 0; i < n; i++) {
      const int pb = A.cbody[i], b1 = pb & 255, b2 = pb >> 8;
      if (b2 == lane) {
        for (int k = 0; k < 18; k++) acc[k] += cw[i][k];
        for (int k = 0; k < 6; k++) acc[18 + k] += cw[i][18 + k];
      }
      if (b1 == lane) {
        for (int k = 0; k < 18; k++) acc[k] -= cw[i][k];
        for (int k = 0; k < 6; k++) acc[18 + k] += cw[i][24 + k];
      }
    }
    for (int k = 0; k < 24; k++) A.dep[lane][k] = acc[k];
  }
  __syncwarp();
}

// limit rows (lane = dof, dofs 6..NV-1): replay with the forward's test, force at the tape's zone; direct tangent
// and velocity cotangents of the dof
template <class SH, class RW>
__device__ __noinline__ int adj_limits(AWorld& s, const SH& W, RW& A, const float* rec, int lane) {
  const float h = G1_TIMESTEP;
  int nlim = 0, mismatch = 0;
  const unsigned below = (1u << lane) - 1u;
  for (int i0 = 0; i0 < NV; i0 += 32) {
    const int i = i0 + lane;
    float dlo = 1.f, dhi = 1.f;
    if (i >= 6 && i < NV) {
      const float q = s.qpos[i + 1];
      dlo = q - ld(g1_dof_range + 2 * i);
      dhi = ld(g1_dof_range + 2 * i + 1) - q;
    }
    const bool on = fminf(dlo, dhi) < 0.f;
    const unsigned bal = __ballot_sync(FULL, on);
    if (on) {
      const int r = nlim + __popc(bal & below);
      const bool active = (W.zone[r >> 5] >> (r & 31)) & 1u;
      if (active) {
        const float pos = fminf(dlo, dhi), sg = dlo < dhi ? 1.f : -1.f;
        const float sr[2] = {ld(g1_jnt_solref), ld(g1_jnt_solref + 1)};
        const float si[5] = {ld(g1_jnt_solimp), ld(g1_jnt_solimp + 1), ld(g1_jnt_solimp + 2),
                             ld(g1_jnt_solimp + 3), ld(g1_jnt_solimp + 4)};
        float kk, bb, imp0, imp, dimp;
        impedance(sr, si, pos, h, &kk, &bb, &imp0);
        impedance_d(si, pos, &imp, &dimp);
        const float iw = ld(g1_dof_invweight0 + i);
        const float R = fmaxf(1e-15f, iw * (1.f - imp) / imp), D = 1.f / R;
        const float dD = R > 1e-15f ? D * D * iw / (imp * imp) : 0.f;
        // psi = (sg lam) (-D) (sg a + b sg v + k imp pos)
        const float lam = A.lam[i], a = s.qacc[i], v = s.qvel[i];
        const float Bt = sg * a + bb * sg * v + kk * imp * pos;
        A.vb[i] += -D * bb * lam;
        const float dpos = -sg * lam * (dD * dimp * Bt + D * kk * (imp + dimp * pos));
        A.qout[i] += sg * dpos;
      }
    }
    nlim += __popc(bal);
  }
  mismatch = nlim != W.nlim_tape;
  __syncwarp();
  return mismatch;
}

// (P . s) of the pose wrench P = (moment about the origin, force) along the motion vector of dof i on body b
__device__ __forceinline__ float wrench_dot(const float* P, const float* w, const float* Xb) {
  float xw[3];
  cross(Xb, w, xw);
  return dot3(P, w) + dot3(P + 3, xw);
}

// The leaf-to-root sweep (lane = body, deepest level first): each body's local reverse of both ID channels (its
// COM acceleration, wrench and inertia), the velocity / acceleration recursion cotangents to its parent, the
// subtree sums, and its dofs' tangent and velocity cotangents
template <class SH, class RW>
__device__ __noinline__ void adj_sweep(AWorld& s, const SH& W, RW& A, int lane) {
  const int b = lane;
  const int depth = b < NB ? ldi(g1_body_depth + b) : -1;
  const int nch = b < NB ? ldi(g1_body_nchild + b) : 0;
  // each body's own terms first, all bodies at once (they need only the replay), kept in registers: its channels'
  // own wrenches (Sown), the velocity / acceleration cotangents it causes, its rotation and COM-point cotangents;
  // the level-by-level sweep then only adds the children's and does the recursion
  float Q[4], X[3], om[3], alA[3], aoA[3], alB[3], aoB[3];
  float omb[3] = {0.f, 0.f, 0.f}, alAb[3] = {0.f, 0.f, 0.f}, aoAb[3] = {0.f, 0.f, 0.f};
  float alBb[3] = {0.f, 0.f, 0.f}, aoBb[3] = {0.f, 0.f, 0.f};
  float S[36], P[6];
  float rho[3] = {0.f, 0.f, 0.f};  // rotation cotangent (a pure moment)
  float cwb[3] = {0.f, 0.f, 0.f};  // cotangent of the COM point
  for (int k = 0; k < 36; k++) S[k] = 0.f;
  for (int k = 0; k < 6; k++) P[k] = 0.f;
  if (b >= 1 && b < NB) {
    for (int k = 0; k < 4; k++) Q[k] = s.Q[b][k];
    for (int k = 0; k < 3; k++) {
      X[k] = s.X[b][k]; om[k] = W.om[b][k]; alA[k] = W.alA[b][k]; aoA[k] = W.aoA[b][k];
      alB[k] = W.alB[b][k]; aoB[k] = W.aoB[b][k];
    }
    // this body's own terms
    {
      float ip[3] = {ld(g1_body_ipos + 3 * b), ld(g1_body_ipos + 3 * b + 1), ld(g1_body_ipos + 3 * b + 2)};
      if (b == G1_TORSO)
        for (int k = 0; k < 3; k++) ip[k] += s.com[k];
      float c[3], cw[3];
      qrot(Q, ip, c);
      for (int k = 0; k < 3; k++) cw[k] = X[k] + c[k];
      const float iq[4] = {ld(g1_body_iquat + 4 * b), ld(g1_body_iquat + 4 * b + 1), ld(g1_body_iquat + 4 * b + 2),
                           ld(g1_body_iquat + 4 * b + 3)};
      float qi[4], Rm[3][3];
      qmul(Q, iq, qi);
      for (int k = 0; k < 3; k++) {
        float e[3] = {0.f, 0.f, 0.f}, col[3];
        e[k] = 1.f;
        qrot(qi, e, col);
        for (int r = 0; r < 3; r++) Rm[r][k] = col[r];
      }
      const float In[3] = {ld(g1_body_inertia + 3 * b), ld(g1_body_inertia + 3 * b + 1),
                           ld(g1_body_inertia + 3 * b + 2)};
      float I[3][3];
      for (int r = 0; r < 3; r++)
        for (int q = 0; q < 3; q++)
          I[r][q] = Rm[r][0] * In[0] * Rm[q][0] + Rm[r][1] * In[1] * Rm[q][1] + Rm[r][2] * In[2] * Rm[q][2];
      auto Iv = [&](const float* x, float* o) {
        for (int r = 0; r < 3; r++) o[r] = I[r][0] * x[0] + I[r][1] * x[1] + I[r][2] * x[2];
      };
      const float m = ld(g1_body_mass + b);
      // ---- channel A: weight -1, motion of lambda
      {
        const float* V = A.VL[b];
        float u1[3], u2[3], u3[3], ac[3], F[3], Iom[3], Ial[3], N[3], t[3];
        cross(alA, c, u1);
        cross(om, c, u2);
        cross(om, u2, u3);
        for (int k = 0; k < 3; k++) { ac[k] = aoA[k] + u1[k] + u3[k]; F[k] = m * ac[k]; }
        Iv(om, Iom);
        Iv(alA, Ial);
        cross(om, Iom, t);
        for (int k = 0; k < 3; k++) N[k] = Ial[k] + t[k];
        // own wrench at the origin into the subtree sum: (N + cw x F, F)
        cross(cw, F, t);
        for (int k = 0; k < 3; k++) { S[k] += N[k] + t[k]; S[3 + k] += F[k]; }
        // cotangents: Fbar = -(V_lin + W x cw), Nbar = -W, cw gets W x F ... (psi_A = -<W_b, V^lambda_b>)
        float Fb[3], Nb[3];
        cross(V, cw, t);
        for (int k = 0; k < 3; k++) { Fb[k] = -(V[3 + k] + t[k]); Nb[k] = -V[k]; }
        cross(V, F, t);
        for (int k = 0; k < 3; k++) cwb[k] += t[k];
        // N = I al + om x (I om)
        float n2[3], Inb[3], In2[3], t2[3];
        Iv(Nb, Inb);
        for (int k = 0; k < 3; k++) alAb[k] += Inb[k];
        cross(Nb, om, n2);  // n . (om x I om) = (n x om) . I om
        Iv(n2, In2);
        cross(Iom, Nb, t);
        cross(Nb, om, t2);
        float Int2[3];
        Iv(t2, Int2);
        for (int k = 0; k < 3; k++) omb[k] += t[k] + Int2[k];
        // rotation of the inertia: n . (I x) -> (I x) x n + (I n) x x
        cross(Ial, Nb, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        cross(Inb, alA, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        cross(Iom, n2, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        cross(In2, om, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        // F = m ac, ac = ao + al x c + om x (om x c)
        float acb[3], cb[3], z[3], zb[3];
        for (int k = 0; k < 3; k++) { acb[k] = m * Fb[k]; aoAb[k] += acb[k]; }
        cross(c, acb, t);
        for (int k = 0; k < 3; k++) alAb[k] += t[k];
        cross(acb, alA, cb);
        cross(om, c, z);
        cross(acb, om, zb);
        cross(z, acb, t);
        for (int k = 0; k < 3; k++) omb[k] += t[k];
        cross(c, zb, t);
        for (int k = 0; k < 3; k++) omb[k] += t[k];
        cross(zb, om, t);
        for (int k = 0; k < 3; k++) cb[k] += t[k];
        cross(c, cb, t);  // c = R ip (relative): a rotation moment
        for (int k = 0; k < 3; k++) rho[k] += t[k];
      }
      // ---- channel B: weight +1, motion of y, om = 0
      {
        const float* V = A.VY[b];
        float u1[3], ac[3], F[3], N[3], t[3];
        cross(alB, c, u1);
        for (int k = 0; k < 3; k++) { ac[k] = aoB[k] + u1[k]; F[k] = m * ac[k]; }
        Iv(alB, N);
        cross(cw, F, t);
        for (int k = 0; k < 3; k++) { S[6 + k] += N[k] + t[k]; S[9 + k] += F[k]; }
        float Fb[3], Nb[3];
        cross(V, cw, t);
        for (int k = 0; k < 3; k++) { Fb[k] = V[3 + k] + t[k]; Nb[k] = V[k]; }
        cross(F, V, t);  // cw gets Fbar-side term: Nbar_O . (cw x F) with Nbar_O = W: d/dcw = F x W
        for (int k = 0; k < 3; k++) cwb[k] += t[k];
        float Inb[3];
        Iv(Nb, Inb);
        for (int k = 0; k < 3; k++) alBb[k] += Inb[k];
        cross(N, Nb, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        cross(Inb, alB, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        float acb[3], cb[3];
        for (int k = 0; k < 3; k++) { acb[k] = m * Fb[k]; aoBb[k] += acb[k]; }
        cross(c, acb, t);
        for (int k = 0; k < 3; k++) alBb[k] += t[k];
        cross(acb, alB, cb);
        cross(c, cb, t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
      }
      // the COM point's cotangent as a force at cw
      float t[3];
      cross(cw, cwb, t);
      for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += cwb[k]; }
    }
  }
  for (int L = MAXD; L >= 1; L--) {
    if (depth == L) {
      const int d = b + 4;  // hinge dof (b >= 2)
      // the deposits, then the inflow from the children: velocity / acceleration cotangents, relative-position
      // forces, subtree sums
      for (int k = 0; k < 18; k++) S[12 + k] = A.dep[b][k];
      for (int k = 0; k < 6; k++) P[k] += A.dep[b][18 + k];
      for (int ci = 0; ci < nch; ci++) {
        const int ch = ldi(g1_body_child + 3 * b + ci);
        for (int k = 0; k < 3; k++) {
          omb[k] += A.up[ch][k]; alAb[k] += A.up[ch][3 + k]; aoAb[k] += A.up[ch][6 + k];
          alBb[k] += A.up[ch][9 + k]; aoBb[k] += A.up[ch][12 + k];
        }
        // the child's relative-position cotangent acts on this body's origin: force -rbar at X
        float rb[3] = {A.up[ch][15], A.up[ch][16], A.up[ch][17]}, t[3];
        cross(X, rb, t);
        for (int k = 0; k < 3; k++) { P[k] -= t[k]; P[3 + k] -= rb[k]; }
        for (int k = 0; k < 36; k++) S[k] += A.sub[ch][k];
      }
      // the velocity / acceleration recursion to the parent (hinge bodies), the dof's terms
      float up[18];
      for (int k = 0; k < 18; k++) up[k] = 0.f;
      if (b >= 2) {
        const int p = ldi(g1_body_parent + b);
        float w[3] = {W.ax[d][0], W.ax[d][1], W.ax[d][2]}, Xp[3], omp[3], alAp[3], alBp[3], r[3];
        for (int k = 0; k < 3; k++) {
          Xp[k] = s.X[p][k]; omp[k] = W.om[p][k]; alAp[k] = W.alA[p][k]; alBp[k] = W.alB[p][k]; r[k] = X[k] - Xp[k];
        }
        const float vd = s.qvel[d], ad = s.qacc[d], xd = W.xa[d];
        float wb[3] = {0.f, 0.f, 0.f}, t[3], z[3], zb[3], rb[3];
        // A: om_b = om_p + w vd; al_b = al_p + om_p x (w vd) + w ad; ao_b = ao_p + al_p x r + om_p x (om_p x r)
        for (int k = 0; k < 3; k++) { up[k] = omb[k]; up[3 + k] = alAb[k]; up[6 + k] = aoAb[k]; }
        for (int k = 0; k < 3; k++) wb[k] += vd * omb[k] + ad * alAb[k];
        float vbar = dot3(w, omb);
        float wv[3] = {w[0] * vd, w[1] * vd, w[2] * vd}, aw[3];
        cross(wv, alAb, t);  // om_p gets (w vd) x albar
        for (int k = 0; k < 3; k++) up[k] += t[k];
        cross(alAb, omp, aw);  // (w vd) gets albar x om_p
        for (int k = 0; k < 3; k++) wb[k] += vd * aw[k];
        vbar += dot3(w, aw);
        cross(r, aoAb, t);
        for (int k = 0; k < 3; k++) up[3 + k] += t[k];
        cross(omp, r, z);
        cross(aoAb, omp, zb);
        cross(z, aoAb, t);
        for (int k = 0; k < 3; k++) up[k] += t[k];
        cross(r, zb, t);
        for (int k = 0; k < 3; k++) up[k] += t[k];
        cross(aoAb, alAp, rb);
        cross(zb, omp, t);
        for (int k = 0; k < 3; k++) rb[k] += t[k];
        // B: al_b = al_p + w xd; ao_b = ao_p + al_p x r
        for (int k = 0; k < 3; k++) { up[9 + k] = alBb[k]; up[12 + k] = aoBb[k]; wb[k] += xd * alBb[k]; }
        cross(r, aoBb, t);
        for (int k = 0; k < 3; k++) up[9 + k] += t[k];
        cross(aoBb, alBp, t);
        for (int k = 0; k < 3; k++) rb[k] += t[k];
        // r = X - Xp: force rbar at X (this body), -rbar at Xp (the parent: up[15..17])
        cross(X, rb, t);
        for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += rb[k]; up[15 + k] = rb[k]; }
        A.vb[d] += vbar;
        // the dof's motion vector s = (w, X x w): sbar = -lam W_A + y W_B + lam G_l + a G_a + v G_v (subtree sums)
        const float lam = A.lam[d], yd = A.y[d];
        float sb[6];
        for (int k = 0; k < 6; k++)
          sb[k] = -lam * S[k] + yd * S[6 + k] + lam * S[12 + k] + ad * S[18 + k] + vd * S[24 + k];
        A.vb[d] += wrench_dot(S + 24, w, X);
        // s depends on w (rotates with the body) and X: wbar += sb_ang + sb_lin x X, X gets w x sb_lin
        cross(sb + 3, X, t);
        for (int k = 0; k < 3; k++) wb[k] += sb[k] + t[k];
        float xf[3];
        cross(w, sb + 3, xf);
        cross(X, xf, t);
        for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += xf[k]; }
        cross(w, wb, t);  // the axis rotates with the body
        for (int k = 0; k < 3; k++) rho[k] += t[k];
        for (int k = 0; k < 3; k++) P[k] += rho[k];
        for (int k = 0; k < 6; k++) S[30 + k] += P[k];
        A.qb[d] += wrench_dot(S + 30, w, X);
      } else {  // the root: its 6 dofs; om_1 = sum_i w_i v_i, al_1 = sum_i w_i a_i (w_i = R e_i: the body's axes)
        float t[3];
        float wbr[3][3];
        for (int i = 0; i < 3; i++) {
          const float* w = W.ax[3 + i];
          A.vb[3 + i] += dot3(w, omb);  // om = sum_i w_i v_i
          for (int k = 0; k < 3; k++)
            wbr[i][k] = s.qvel[3 + i] * omb[k] + s.qacc[3 + i] * alAb[k] + W.xa[3 + i] * alBb[k];
        }
        for (int i = 0; i < 6; i++) {
          const float lam = A.lam[i], yd = A.y[i], ad = s.qacc[i], vd = s.qvel[i];
          float sb[6];
          for (int k = 0; k < 6; k++)
            sb[k] = -lam * S[k] + yd * S[6 + k] + lam * S[12 + k] + ad * S[18 + k] + vd * S[24 + k];
          if (i < 3) {
            A.vb[i] += S[27 + i];  // s = (0, e_i)
          } else {
            const float* w = W.ax[i];
            A.vb[i] += wrench_dot(S + 24, w, X);
            cross(sb + 3, X, t);
            for (int k = 0; k < 3; k++) wbr[i - 3][k] += sb[k] + t[k];
            float xf[3];
            cross(w, sb + 3, xf);
            cross(X, xf, t);
            for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += xf[k]; }
          }
        }
        for (int i = 0; i < 3; i++) {
          cross(W.ax[3 + i], wbr[i], t);
          for (int k = 0; k < 3; k++) rho[k] += t[k];
        }
        for (int k = 0; k < 3; k++) P[k] += rho[k];
        for (int k = 0; k < 6; k++) S[30 + k] += P[k];
        for (int i = 0; i < 3; i++) A.qb[i] += S[33 + i];
        for (int i = 3; i < 6; i++) A.qb[i] += wrench_dot(S + 30, W.ax[i], X);
      }
      for (int k = 0; k < 36; k++) A.sub[b][k] = S[k];
      for (int k = 0; k < 18; k++) A.up[b][k] = up[k];
    }
    __syncwarp();
  }
}

// dst[0..NTRI) <- src (a factor from the tape): each lane's 20 loads issued before its first store, so the copy
// waits for one memory round trip instead of one per element
__device__ __forceinline__ void copy_factor(float* dst, const float* src, int lane) {
  constexpr int R = (NTRI + 31) / 32;
  float v[R];
#pragma unroll
  for (int q = 0; q < R; q++) v[q] = lane + 32 * q < NTRI ? __ldg(src + lane + 32 * q) : 0.f;
#pragma unroll
  for (int q = 0; q < R; q++)
    if (lane + 32 * q < NTRI) dst[lane + 32 * q] = v[q];
}

// dst[0..NTRI) <- the tape's tree-block factor: its NTB pattern entries from src, zeros elsewhere (written here when
// `zero`, else already there: nothing else writes outside the pattern); each lane's loads issued before its stores
__device__ __forceinline__ void copy_factor_tb(float* dst, const float* src, int lane, bool zero) {
  constexpr int R = (NTB + 31) / 32;
  float v[R];
#pragma unroll
  for (int q = 0; q < R; q++) v[q] = lane + 32 * q < NTB ? __ldg(src + lane + 32 * q) : 0.f;
  if (zero) {
    for (int e = lane; e < NTRI; e += 32) dst[e] = 0.f;
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < R; q++)
    if (lane + 32 * q < NTB) dst[g_tb_index.e[lane + 32 * q]] = v[q];
}

// One substep of the adjoint from its tape record rec: adj_record (the record's state into s and W), the replay
// (adj_replay: poses, velocities and accelerations, the motions of a* and v, the geom poses and contact rows), and for
// the cotangent (A.qout / A.vb in: the substep output's tangent and velocity cotangents; out: the input's, A.ub
// accumulating the ctrl gradient) adj_row_solve (the integrator and both solves, each factor copied into the state's
// scratch just before its solve, L_Q rebuilt there from a compact record) and adj_row_rest. block_sync: every warp of
// the block calls adj_substep together; a block barrier before the limit rows and the sweep re-aligns the worlds
// after their contact loops (different lengths): 1.06 -> 1.02 ms at B = 4096
template <class SH>
__device__ __forceinline__ void adj_record(AWorld& s, SH& W, const float* rec, int lane) {
  for (int i = lane; i < NQ; i += 32) s.qpos[i] = rec[T_QPOS + i];
  for (int i = lane; i < NV; i += 32) {
    s.qvel[i] = rec[T_QVEL + i];
    s.qacc[i] = rec[T_ASTAR + i];
    W.aadv[i] = rec[T_AADV + i];
    W.xa[i] = s.qacc[i] - W.aadv[i];
  }
  const unsigned hdr = __float_as_uint(rec[T_HDR]);
  if (lane == 0) {
    s.ncon = hdr & 255u;
    s.nefc = (hdr >> 8) & 255u;
    W.nlim_tape = (hdr >> 16) & 255u;
    W.clamp_lo = __float_as_uint(rec[T_CLAMP]);
    for (int k = 0; k < NEFC / 32; k++) W.zone[k] = __float_as_uint(rec[T_ZONE + k]);
    W.clamp_hi = __float_as_uint(rec[T_CLAMP + 1]);
  }
  for (int c = lane; c < MAXCON; c += 32) {
    const unsigned e = (__float_as_uint(rec[T_CON + c / 2]) >> (16 * (c & 1))) & 0xffffu;
    s.con_pair[c] = (int)(e & 511u);
    s.con_slot[c] = (unsigned char)(e >> 9);
  }
  __syncwarp();
}

// the geom poses from the replayed body poses (lane = geom)
template <class SH>
__device__ __forceinline__ void adj_replay_geoms(const AWorld& s, SH& W, int lane) {
  for (int g = lane; g < NG; g += 32) {
    const int b = ldi(g1_geom_body + g);
    const float gp[3] = {ld(g1_geom_pos + 3 * g), ld(g1_geom_pos + 3 * g + 1), ld(g1_geom_pos + 3 * g + 2)};
    const float gq[4] = {ld(g1_geom_quat + 4 * g), ld(g1_geom_quat + 4 * g + 1), ld(g1_geom_quat + 4 * g + 2),
                         ld(g1_geom_quat + 4 * g + 3)};
    float t[3];
    qrot(s.Q[b], gp, t);
    for (int k = 0; k < 3; k++) W.col.gx[g][k] = s.X[b][k] + t[k];
    qmul(s.Q[b], gq, W.col.gq[g]);
  }
}

// the contacts' rows: the same numbering as the forward (limit rows first; lane = contact)
template <class SH>
__device__ __forceinline__ void adj_replay_rows(AWorld& s, const SH& W, int lane) {
  const int ncon = s.ncon;
  int r0 = W.nlim_tape;
  for (int c0 = 0; c0 < ncon; c0 += 32) {
    const int c = c0 + lane;
    const int want = c < ncon ? (ldi(g1_pair_dim + s.con_pair[c]) == 3 ? 4 : 1) : 0;
    int incl = want;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += t;
    }
    const int first = r0 + incl - want;
    if (c < ncon) {
      s.con_row0[c] = (unsigned char)min(first, 255);
      s.con_nrow[c] = (unsigned char)max(0, min(want, NEFC - first));
    }
    r0 += __shfl_sync(FULL, incl, 31);
  }
}

template <class SH>
__device__ __forceinline__ void adj_replay(AWorld& s, SH& W, int lane) {
  // the replay: poses and both channels; the motions of a* and v; the geom poses and the contacts' rows
  adj_replay_kin(s, W, lane);
  adj_motion(s, W, s.qacc, W.VA, lane);
  adj_motion(s, W, s.qvel, W.VV, lane);
  adj_replay_geoms(s, W, lane);
  adj_replay_rows(s, W, lane);
  __syncwarp();
}

// L_Q from the replayed poses (the compact tape stores none): the forward's mass matrix (mass_and_force: each body's
// spatial inertia about the pelvis origin O summed over its subtree, M_ij = s_j . I s_i over the ancestor dofs j of
// dof i, the armature on the diagonal) and its tree-block factor with h kv, into L / dinv. M and Ic: scratch; lane =
// body, then dof.
template <class SH>
__device__ __noinline__ void adj_mass_factor(const AWorld& s, const SH& W, float* M, float (*Ic)[10], float* L,
                                             float* dinv, int lane) {
  const float O[3] = {s.X[1][0], s.X[1][1], s.X[1][2]};
  const int b = lane;
  if (b >= 1 && b < NB) {
    float ip[3] = {ld(g1_body_ipos + 3 * b), ld(g1_body_ipos + 3 * b + 1), ld(g1_body_ipos + 3 * b + 2)};
    if (b == G1_TORSO)
      for (int k = 0; k < 3; k++) ip[k] += s.com[k];
    float c[3], qi[4], Rm[3][3];
    qrot(s.Q[b], ip, c);
    const float iq[4] = {ld(g1_body_iquat + 4 * b), ld(g1_body_iquat + 4 * b + 1), ld(g1_body_iquat + 4 * b + 2),
                         ld(g1_body_iquat + 4 * b + 3)};
    qmul(s.Q[b], iq, qi);
    for (int k = 0; k < 3; k++) {
      float e[3] = {0.f, 0.f, 0.f}, col[3];
      e[k] = 1.f;
      qrot(qi, e, col);
      for (int r = 0; r < 3; r++) Rm[r][k] = col[r];
    }
    const float In[3] = {ld(g1_body_inertia + 3 * b), ld(g1_body_inertia + 3 * b + 1),
                         ld(g1_body_inertia + 3 * b + 2)};
    float I[3][3];
    for (int r = 0; r < 3; r++)
      for (int q = r; q < 3; q++) {
        const float v = Rm[r][0] * In[0] * Rm[q][0] + Rm[r][1] * In[1] * Rm[q][1] + Rm[r][2] * In[2] * Rm[q][2];
        I[r][q] = v; I[q][r] = v;
      }
    const float m = ld(g1_body_mass + b);
    float cO[3];
    for (int k = 0; k < 3; k++) cO[k] = s.X[b][k] + c[k] - O[k];
    const float cc = dot3(cO, cO);
    float* J = Ic[b];
    J[0] = I[0][0] + m * (cc - cO[0] * cO[0]);
    J[1] = I[1][1] + m * (cc - cO[1] * cO[1]);
    J[2] = I[2][2] + m * (cc - cO[2] * cO[2]);
    J[3] = I[0][1] - m * cO[0] * cO[1];
    J[4] = I[0][2] - m * cO[0] * cO[2];
    J[5] = I[1][2] - m * cO[1] * cO[2];
    J[6] = m * cO[0]; J[7] = m * cO[1]; J[8] = m * cO[2]; J[9] = m;
  }
  __syncwarp();
  const int depth = b < NB ? ldi(g1_body_depth + b) : -1, nch = b < NB ? ldi(g1_body_nchild + b) : 0;
  for (int lv = MAXD - 1; lv >= 1; lv--) {
    if (depth == lv && nch > 0) {
      float J[10];
      for (int k = 0; k < 10; k++) J[k] = Ic[b][k];
      for (int ci = 0; ci < nch; ci++) {
        const int ch = ldi(g1_body_child + 3 * b + ci);
        for (int k = 0; k < 10; k++) J[k] += Ic[ch][k];
      }
      for (int k = 0; k < 10; k++) Ic[b][k] = J[k];
    }
    __syncwarp();
  }
  for (int e = lane; e < NTRIP / 4; e += 32) reinterpret_cast<float4*>(M)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  // dof i's motion about O: translations (0, e_i), the pelvis's rotations (w, 0), hinges (w, w x (O - X_b))
  auto motion = [&](int i, float* w, float* v) {
    for (int k = 0; k < 3; k++) { w[k] = i < 3 ? 0.f : W.ax[i][k]; v[k] = i < 3 && k == i ? 1.f : 0.f; }
    if (i >= 6) {
      const int bb = i - 4;
      const float r[3] = {O[0] - s.X[bb][0], O[1] - s.X[bb][1], O[2] - s.X[bb][2]};
      cross(w, r, v);
    }
  };
  for (int i = lane; i < NV; i += 32) {
    const int bi = ldi(g1_dof_body + i);
    float w[3], v[3], n[3], f[3];
    motion(i, w, v);
    apply_inertia(Ic[bi], w, v, n, f);
    unsigned long long anc = g1_body_dofmask[bi] & ((1ull << i) - 1ull);
    while (anc) {
      const int j = __ffsll((long long)anc) - 1;
      anc &= anc - 1ull;
      float wj[3], vj[3];
      motion(j, wj, vj);
      M[TRI(i, j)] = dot3(wj, n) + dot3(vj, f);
    }
    M[TRI(i, i)] = dot3(w, n) + dot3(v, f) + ld(g1_dof_armature + i);
  }
  __syncwarp();
  tb_factor(M, true, L, dinv, lane);
}

// full: rec holds L_Q (a full record), else it is rebuilt from the replayed poses (adj_replay_kin must have run)
template <class SH, class RW>
__device__ __forceinline__ void adj_row_solve(AWorld& s, const SH& W, RW& A, const float* rec, bool full, int lane) {
  const float h = G1_TIMESTEP;
  PROF_START(A);
  // A1: the integrator. v' = v + h a_adv; root rotation: q' = q exp(h w' / 2). The input tangent gets qbar' (kept in
  // qout), its rotation R(h w') qbar'_rot
  {
    for (int i = lane; i < NV; i += 32) {
      float vt = A.vb[i];
      if (i < 3 || i >= 6) vt += h * A.qout[i];
      A.y[i] = vt;  // (vbar'_tot; the rotation's part is added by lane 0 below)
    }
    __syncwarp();
    if (lane == 0) {
      const float w[3] = {s.qvel[3] + h * W.aadv[3], s.qvel[4] + h * W.aadv[4], s.qvel[5] + h * W.aadv[5]};
      const float tb[3] = {A.qout[3], A.qout[4], A.qout[5]};
      const float ph[3] = {h * w[0], h * w[1], h * w[2]};
      const float th = sqrtf(dot3(ph, ph));
      // R(phi) tb and J_r(phi)' tb; J_r = I - (1 - cos th) / th^2 [phi]x + (th - sin th) / th^3 [phi]x^2
      float c1, c2;
      if (th < 1e-3f) { c1 = 0.5f - th * th / 24.f; c2 = 1.f / 6.f - th * th / 120.f; }
      else { float sn, cs; sincosf(th, &sn, &cs); c1 = (1.f - cs) / (th * th); c2 = (th - sn) / (th * th * th); }
      float pt[3], ppt[3];
      cross(ph, tb, pt);
      cross(ph, pt, ppt);
      // J_r' tb = tb + c1 phi x tb + c2 phi x (phi x tb)  ([phi]x' = -[phi]x)
      for (int k = 0; k < 3; k++) A.y[3 + k] += h * (tb[k] + c1 * pt[k] + c2 * ppt[k]);
      // R(phi) tb (rotation by angle th about phi): Rodrigues
      float sn = 0.f, omc = 0.f;
      if (th < 1e-3f) { sn = 1.f - th * th / 6.f; omc = 0.5f - th * th / 24.f; }
      else { float s_, c_; sincosf(th, &s_, &c_); sn = s_ / th; omc = (1.f - c_) / (th * th); }
      for (int k = 0; k < 3; k++) A.qout[3 + k] = tb[k] + sn * pt[k] + omc * ppt[k];
    }
    __syncwarp();
    for (int i = lane; i < NV; i += 32) {
      A.vb[i] = A.y[i];      // v' = v + h a_adv: the input velocity gets vbar'_tot
      A.y[i] = h * A.y[i];   // abar_adv
    }
    __syncwarp();
  }
  PROF(A, 0);
  // y = (M + h kv)^-1 abar_adv with L_Q; abar* = abar_adv - h kv y (each factor copied in just before its solve)
  float* L = A.L;
  float* dinv = A.dinv;
  if (full) {
    copy_factor_tb(L, rec + T_LQ, lane, true);
    for (int i = lane; i < NV; i += 32) dinv[i] = rec[T_DINVQ + i];
  } else {
    adj_mass_factor(s, W, A.M, A.Ic, L, dinv, lane);
  }
  for (int i = lane; i < NV; i += 32) A.lam[i] = A.y[i];
  __syncwarp();
  chol_solve<true>(L, dinv, A.y, lane);  // L_Q is in tree-block order
  for (int i = lane; i < NV; i += 32) A.lam[i] -= h * ld(g1_dof_kv + i) * A.y[i];
  // A2: lambda = H^-1 abar* with L_H
  __syncwarp();
  copy_factor(L, rec + T_LH, lane);
  for (int i = lane; i < NV; i += 32) dinv[i] = rec[T_DINVH + i];
  __syncwarp();
  chol_solve(L, dinv, A.lam, lane);
  PROF(A, 1);
}

template <class SH, class RW>
__device__ __forceinline__ int adj_row_rest(AWorld& s, const SH& W, RW& A, const float* rec, int clamp_kv,
                                            float clamp_soft, float (*cw)[30], int lane, bool block_sync) {
  int flags = 0;
  // A3: the motions of lambda and y (the replay and those of a*, v are shared)
  adj_motion(s, W, A.lam, A.VL, lane);
  adj_motion(s, W, A.y, A.VY, lane);
  for (int b = lane; b < NB; b += 32)
    for (int k = 0; k < 24; k++) A.dep[b][k] = 0.f;
  PROF(A, 2);
  __syncwarp();
  PROF(A, 3);
  int mism = 0;
  for (int c0 = 0; c0 < s.ncon; c0 += 32) {
    mism |= adj_contacts(s, W, A, rec, cw, c0, lane);
    adj_contact_deposit(s, A, cw, c0, lane);
  }
  if (__any_sync(FULL, mism)) flags |= ADJ_REPLAY_MISMATCH;
  PROF(A, 4);
  // A6: the limit rows; actuators
  if (block_sync) __syncthreads();
  if (adj_limits(s, W, A, rec, lane)) flags |= ADJ_REPLAY_MISMATCH;
  for (int i = lane; i < NV; i += 32) {
    if (i < 6) continue;
    const float lam = A.lam[i], kp = ld(g1_dof_kp + i), kv = ld(g1_dof_kv + i);
    const bool clamped = i < 32 ? (W.clamp_lo >> i) & 1u : (W.clamp_hi >> (i - 32)) & 1u;
    float wq = clamped ? 0.f : 1.f, wv = clamped ? (clamp_kv == 0 ? 1.f : 0.f) : 1.f;
    if (clamped && clamp_kv == 2 && clamp_soft > 0.f) {
      const float f = kp * (W.u[i - 6] - s.qpos[i + 1]) - kv * s.qvel[i], lim = ld(g1_dof_frclim + i);
      const float o = fmaxf(0.f, (fabsf(f) - lim) / lim);
      wq = wv = __expf(-o / clamp_soft);
    }
    A.qout[i] += -kp * lam * wq;
    A.vb[i] += -kv * lam * wv;
    A.ub[i - 6] += kp * lam * wq;
  }
  __syncwarp();
  // A7: the sweep
  for (int i = lane; i < NV; i += 32) A.qb[i] = 0.f;
  __syncwarp();
  PROF(A, 5);
  adj_sweep(s, W, A, lane);
  PROF(A, 6);
  // A8: the input state's tangent cotangent
  for (int i = lane; i < NV; i += 32) A.qout[i] = A.qb[i] + A.qout[i];
  __syncwarp();
  return flags;
}

// the adjoint's substep (one cotangent per world): both parts in one warp, the factors copied as they are needed
// full: a full record (else compact: the poses are replayed first, for the rebuilt L_Q)
__device__ __forceinline__ int adj_substep(AWorld& s, Adj& A, const float* rec, bool full, int clamp_kv,
                                           float clamp_soft, float (*cw)[30], int lane, bool block_sync = false) {
  adj_record(s, A, rec, lane);
  if (full) {
    adj_row_solve(s, A, A, rec, true, lane);
    adj_replay(s, A, lane);
  } else {
    adj_replay_kin(s, A, lane);
    adj_row_solve(s, A, A, rec, false, lane);
    adj_motion(s, A, s.qacc, A.VA, lane);
    adj_motion(s, A, s.qvel, A.VV, lane);
    adj_replay_geoms(s, A, lane);
    adj_replay_rows(s, A, lane);
    __syncwarp();
  }
  return adj_row_rest(s, A, A, rec, clamp_kv, clamp_soft, cw, lane, block_sync);
}

}  // namespace nbg1
