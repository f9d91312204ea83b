// The step Jacobian as one adjoint with 70 right-hand sides per world: lane = right-hand side.
//
// The VJP of a substep is linear in its cotangent, and everything it multiplies the cotangent with (the tape's
// factors, the replayed poses and motions, the contacts' geometry, frames and impedances, the actuators' clamps) is
// the same for every cotangent of a record. So one block per world prepares those once per record, cooperatively,
// into shared memory (JRec), and then every lane carries one cotangent through the substep with plain scalar code:
// the integrator, the two triangular solves (factor entries read as broadcasts), the limit and actuator terms, and
// one leaf-to-root pass over the bodies that applies the contacts at their bodies and reverses both ID channels. The
// right-hand sides are the tangent basis of the output (q' tangent 0..34, v' 35..69); the 71 output rows (qpos' in
// qpos form, qvel') are formed from them at the end (the quaternion rows as combinations of the three rotation
// cotangents). Same mathematics as the one-cotangent adjoint (nb_g1_adjoint.cuh), reordered for lanes over
// cotangents:
//  * a contact's cotangent terms are linear in lambda's relative motion between its two bodies, dV (6): the record's
//    preparation evaluates contact_terms on the 6 unit dV and keeps the 6-column matrices of G(a*) and of both pose
//    wrenches (G(v) = b G(a*), G(lambda) does not depend on the cotangent and goes into a shared subtree sum);
//  * the own wrenches of both ID channels and G(lambda) enter each dof's terms only through subtree sums, which do
//    not depend on the cotangent either: computed once per record;
//  * the pass visits bodies from the last to the first: a body's motion vectors of lambda and y follow from its
//    child's by removing the child's dof (V_b = V_c - s_c x_c) when the child was visited just before it, else from
//    a sum over its path (a self contact's relative motion: from the dofs between its two bodies, the same bits at
//    both); what a body hands its parent (the recursion's cotangents and the three per-cotangent
//    subtree sums) is carried in registers to a parent visited next, or parked in one per-lane slot (the G1's
//    branch points: the torso's second arm, the pelvis's second and third chains; the upload checks that one slot
//    suffices).
// Reference: OamIcs/NablaEngine scripts/paper_bench/ours.py:99-110 (the Jacobian as 71 backward calls).
#pragma once
#include "nb_g1_adjoint.cuh"

namespace nbg1 {

constexpr int JNR = 2 * NV;   // right-hand sides per world
constexpr int JWARPS = 3;     // warps per block (lane = right-hand side j = 32 warp + lane; j >= JNR: spare lanes)
constexpr int JS = JNR + 2;   // the per-lane arrays' stride: the 70 right-hand sides and 2 spare columns, on which
                              // the spare lanes run (zero cotangents: their arithmetic stays zero)
constexpr int JTHREADS = 32 * JWARPS;
static_assert(JTHREADS >= MAXCON, "one thread per contact in the record's preparation");

// per body (1 .. NB - 1), the same for every cotangent of the record. Every 3-vector sits in a 16-byte slot and every
// 6-vector in two, so that the per-cotangent pass reads each with 128-bit broadcast loads (jv3, jv6).
struct __align__(16) JBody {
  float cw[4], c[4];                 // the COM (world), its offset from the body origin; c[3]: the mass
  float I[8];                        // the inertia at the COM in the world frame: xx, yy, zz, xy, xz, yz
  float FA[4], Iom[4], Ial[4];       // channel A: m ac, I om, I al
  float om[4], alA[4], alB[4];       // the replayed angular velocity and both channels' angular accelerations
  float FB[4], NBc[4];               // channel B: m ac, I al
  float X[4], w[4], r[4];            // body origin, hinge axis (world), origin relative to the parent's
  float SWA[8], SWB[8], SGL[8];      // subtree sums: both channels' own wrenches and G(lambda), at the world origin
};
__device__ __forceinline__ void jv3(const float* p, float* o) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z;
}
__device__ __forceinline__ void jv6(const float* p, float* o) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y;
}
// per contact: the 6-column matrices of its cotangent terms in dV (row-major 6 x 6)
struct JCon {
  float Ga[36], P2[36], P1[36];     // G(a*) (on body 2; -G on body 1), the pose wrenches of body 2 and body 1
  float GL[6];                      // G(lambda), cotangent-independent
  float bb;                         // the rows' damping: G(v) = bb G(a*)
  int b1, b2;
};
struct __align__(16) JRec {
  float LQ[NTRIP], LH[NTRIP];       // the tape's factors: L_Q (tree-block order, zeros off its pattern), L_H
  float dinvQ[NV + 1], dinvH[NV + 1];
  float S6[NV][8];                  // each dof's motion vector (angular, linear at the world origin; 2 slots)
  float vd[NV], ad[NV], xd[NV];     // qvel, a* and a* - a_adv of the record
  float dcq[NV], dcv[NV], dcu[NV];  // limit and actuator terms: tangent, velocity and ctrl cotangents per lambda_i
  float A1[9], A2[9];               // the root rotation's integrator: J_r(h w')' and R(h w') (row-major)
  JBody body[NB];
  JCon con[MAXCON];
  unsigned char cfirst[NB + 1], cmem[2 * MAXCON];  // each body's contacts (as body 1 or body 2)
  int ncon, flags;
};
// per right-hand side (column j of each row of the arrays): lambda, y, the cotangents of q (tangent) and v, the ctrl
// gradient and the parked hand-over. The preparation's scratch (the replayed record: AWorld, AdjShared) shares the
// space of lambda and y, which the cotangents write only after it.
constexpr int JO_LAM = 0, JO_Y = NV, JO_Q = 2 * NV, JO_V = 3 * NV, JO_U = 4 * NV, JO_SLOT = 4 * NV + NU;
constexpr int JSLOT = 36, JRHS_ROWS = JO_SLOT + JSLOT;
struct JPrep { AWorld s; AdjShared W; float M[NTRIP]; float Ic[NB][10]; };  // (M, Ic: a compact record's L_Q)
static_assert(sizeof(JPrep) <= sizeof(float) * 2 * NV * JS, "the preparation's scratch fits lambda and y");
static_assert(offsetof(JPrep, M) % 16 == 0 && offsetof(JRec, LQ) % 16 == 0, "written as float4 by adj_mass_factor");
static_assert(offsetof(JRec, S6) % 16 == 0 && offsetof(JRec, body) % 16 == 0, "read as float4 (jv3, jv6)");
struct __align__(16) JBlock {
  JRec R;
  union {
    float rhs[JRHS_ROWS * JS];
    JPrep prep;
  };
};

// ---- the record's preparation (all threads of the block; t = threadIdx.x) ------------------------------------------
// 1: the record's state (warp 0), the factors (warp 1), the dofs' q, a*, a* - a_adv and the integrator's matrices
// (warp 2); 2: the replay (warp 0), the limit and actuator coefficients (warp 1), each body's contact list (warp 2);
// 3: the contacts' matrices (thread = contact), then the bodies' and dofs' terms; 4: G(lambda) onto the bodies and
// the shared subtree sums (warp 0)
__device__ __forceinline__ void jac_prep_state(JBlock& B, const float* rec, bool full, const float* fric_w,
                                               const float* com_w, const float* ctrl_w, int t) {
  JRec& R = B.R;
  AWorld& s = B.prep.s;
  AdjShared& W = B.prep.W;
  const int warp = t >> 5, lane = t & 31;
  const float h = G1_TIMESTEP;
  if (warp == 0) {
    adj_record(s, W, rec, lane);
    if (lane == 0) { s.fric = *fric_w; R.ncon = s.ncon; }
    if (lane < 3) s.com[lane] = com_w[lane];
    for (int i = lane; i < NU; i += 32) W.u[i] = ctrl_w ? ctrl_w[i] : 0.f;
  } else if (warp == 1) {
    if (full) {  // (a compact record's L_Q is rebuilt from the replayed poses in step 3)
      copy_factor_tb(R.LQ, rec + T_LQ, lane, false);  // (entries off L_Q's pattern: zeroed once)
      for (int i = lane; i < NV; i += 32) R.dinvQ[i] = rec[T_DINVQ + i];
    }
    copy_factor(R.LH, rec + T_LH, lane);
    for (int i = lane; i < NV; i += 32) R.dinvH[i] = rec[T_DINVH + i];
  } else {
    for (int i = lane; i < NV; i += 32) {
      R.vd[i] = rec[T_QVEL + i];
      R.ad[i] = rec[T_ASTAR + i];
      R.xd[i] = R.ad[i] - rec[T_AADV + i];
    }
    if (lane == 0) {
      // q' = q exp(h w' / 2): J_r(phi)' = I + c1 [phi]x + c2 [phi]x^2, R(phi) = I + sn [phi]x + omc [phi]x^2
      const float ph[3] = {h * (rec[T_QVEL + 3] + h * rec[T_AADV + 3]), h * (rec[T_QVEL + 4] + h * rec[T_AADV + 4]),
                           h * (rec[T_QVEL + 5] + h * rec[T_AADV + 5])};
      const float th = sqrtf(dot3(ph, ph));
      float c1, c2, sn, omc;
      if (th < 1e-3f) {
        c1 = 0.5f - th * th / 24.f; c2 = 1.f / 6.f - th * th / 120.f;
        sn = 1.f - th * th / 6.f; omc = 0.5f - th * th / 24.f;
      } else {
        float sv, cv;
        sincosf(th, &sv, &cv);
        c1 = (1.f - cv) / (th * th); c2 = (th - sv) / (th * th * th);
        sn = sv / th; omc = (1.f - cv) / (th * th);
      }
      const float K[9] = {0.f, -ph[2], ph[1], ph[2], 0.f, -ph[0], -ph[1], ph[0], 0.f};  // K v = phi x v
      for (int i = 0; i < 3; i++)
        for (int k = 0; k < 3; k++) {
          float k2 = 0.f;
          for (int q = 0; q < 3; q++) k2 += K[3 * i + q] * K[3 * q + k];
          const float e = i == k ? 1.f : 0.f;
          R.A1[3 * i + k] = e + c1 * K[3 * i + k] + c2 * k2;
          R.A2[3 * i + k] = e + sn * K[3 * i + k] + omc * k2;
        }
    }
  }
}

// the limit rows' and actuators' cotangent terms per lambda_i (one warp): tangent dcq, velocity dcv, ctrl dcu
__device__ __forceinline__ void jac_prep_dofs(JRec& R, const AWorld& s, const AdjShared& W, float clamp_soft,
                                              int clamp_kv, int lane) {
  const float h = G1_TIMESTEP;
  int nlim = 0;
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
    float cq = 0.f, cv = 0.f, cu = 0.f;
    if (on) {  // psi = (sg lam) (-D) (sg a + b sg v + k imp pos), at the tape's zone
      const int r = nlim + __popc(bal & below);
      if ((W.zone[r >> 5] >> (r & 31)) & 1u) {
        const float pos = fminf(dlo, dhi), sg = dlo < dhi ? 1.f : -1.f;
        const float sr[2] = {ld(g1_jnt_solref), ld(g1_jnt_solref + 1)};
        const float si[5] = {ld(g1_jnt_solimp), ld(g1_jnt_solimp + 1), ld(g1_jnt_solimp + 2),
                             ld(g1_jnt_solimp + 3), ld(g1_jnt_solimp + 4)};
        float kk, bb, imp0, imp, dimp;
        impedance(sr, si, pos, h, &kk, &bb, &imp0);
        impedance_d(si, pos, &imp, &dimp);
        const float iw = ld(g1_dof_invweight0 + i);
        const float Rr = fmaxf(1e-15f, iw * (1.f - imp) / imp), D = 1.f / Rr;
        const float dD = Rr > 1e-15f ? D * D * iw / (imp * imp) : 0.f;
        const float Bt = sg * s.qacc[i] + bb * sg * s.qvel[i] + kk * imp * pos;
        cv = -D * bb;
        cq = -(dD * dimp * Bt + D * kk * (imp + dimp * pos));
      }
    }
    nlim += __popc(bal);
    if (i >= 6 && i < NV) {  // the PD actuator (clamp_kv: the derivative on clamped dofs, as in adj_row_rest)
      const float kp = ld(g1_dof_kp + i), kv = ld(g1_dof_kv + i);
      const bool clamped = i < 32 ? (W.clamp_lo >> i) & 1u : (W.clamp_hi >> (i - 32)) & 1u;
      float wq = clamped ? 0.f : 1.f, wv = clamped ? (clamp_kv == 0 ? 1.f : 0.f) : 1.f;
      if (clamped && clamp_kv == 2 && clamp_soft > 0.f) {
        const float f = kp * (W.u[i - 6] - s.qpos[i + 1]) - kv * s.qvel[i], lim = ld(g1_dof_frclim + i);
        const float o = fmaxf(0.f, (fabsf(f) - lim) / lim);
        wq = wv = __expf(-o / clamp_soft);
      }
      cq += -kp * wq;
      cv += -kv * wv;
      cu = kp * wq;
    }
    if (i < NV) { R.dcq[i] = cq; R.dcv[i] = cv; R.dcu[i] = cu; }
  }
  if (lane == 0 && nlim != W.nlim_tape) atomicOr(&R.flags, ADJ_REPLAY_MISMATCH);
}

// each body's contacts (one warp, lane = body): those with the body as body 1 or body 2, in contact order
__device__ __forceinline__ void jac_prep_lists(JRec& R, const AWorld& s, int lane) {
  const int ncon = s.ncon, b = lane;
  int n = 0;
  for (int c = 0; c < ncon; c++) {
    const int pr = s.con_pair[c];
    const int b1 = ldi(g1_geom_body + ldi(g1_pair_g1 + pr)), b2 = ldi(g1_geom_body + ldi(g1_pair_g2 + pr));
    n += b >= 1 && b < NB && (b1 == b || b2 == b);
  }
  int incl = n;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += v;
  }
  int first = incl - n;  // (lane NB, no body: the total)
  if (b <= NB) R.cfirst[b] = (unsigned char)first;
  for (int c = 0; c < ncon && n > 0; c++) {
    const int pr = s.con_pair[c];
    const int b1 = ldi(g1_geom_body + ldi(g1_pair_g1 + pr)), b2 = ldi(g1_geom_body + ldi(g1_pair_g2 + pr));
    if (b1 == b || b2 == b) R.cmem[first++] = (unsigned char)c;
  }
}

// item i < 3 ncon: contact i / 3's matrix columns 2 (i % 3) and 2 (i % 3) + 1, from its terms at those unit dV (the
// contact's cotangent-independent part is computed by each of its three items)
__device__ __forceinline__ void jac_prep_contact(JRec& R, const AWorld& s, const AdjShared& W, int normal, int i) {
  const int c = i / 3, e0 = 2 * (i - 3 * c);
  JCon& C = R.con[c];
  const int mism = contact_terms<2>(
      s, W, c, normal,
      [&](int e, int b1, int b2, float* dV) {
        for (int k = 0; k < 6; k++) dV[k] = k == e0 + e ? 1.f : 0.f;
        if (e0 + e == 0) { C.b1 = b1; C.b2 = b2; }
      },
      [&](int e, const float* o, float bb) {
        const int col = e0 + e;
        for (int k = 0; k < 6; k++) {
          C.Ga[6 * k + col] = o[6 + k];
          C.P2[6 * k + col] = o[18 + k];
          C.P1[6 * k + col] = o[24 + k];
        }
        if (col == 0) {
          for (int k = 0; k < 6; k++) C.GL[k] = o[k];
          C.bb = bb;
        }
      });
  if (mism && e0 == 0) atomicOr(&R.flags, ADJ_REPLAY_MISMATCH);
}

// thread b in 1..NB-1: body b's cotangent-independent terms (the own terms of both ID channels, as adj_sweep)
__device__ __forceinline__ void jac_prep_body(JRec& R, const AWorld& s, const AdjShared& W, int b) {
  JBody& J = R.body[b];
  float Q[4], X[3], om[3], alA[3], aoA[3], alB[3], aoB[3];
  for (int k = 0; k < 4; k++) Q[k] = s.Q[b][k];
  for (int k = 0; k < 3; k++) {
    X[k] = s.X[b][k]; om[k] = W.om[b][k]; alA[k] = W.alA[b][k]; aoA[k] = W.aoA[b][k];
    alB[k] = W.alB[b][k]; aoB[k] = W.aoB[b][k];
  }
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
  const float In[3] = {ld(g1_body_inertia + 3 * b), ld(g1_body_inertia + 3 * b + 1), ld(g1_body_inertia + 3 * b + 2)};
  float I[3][3];
  for (int r = 0; r < 3; r++)
    for (int q = 0; q < 3; q++)
      I[r][q] = Rm[r][0] * In[0] * Rm[q][0] + Rm[r][1] * In[1] * Rm[q][1] + Rm[r][2] * In[2] * Rm[q][2];
  auto Iv = [&](const float* x, float* o) {
    for (int r = 0; r < 3; r++) o[r] = I[r][0] * x[0] + I[r][1] * x[1] + I[r][2] * x[2];
  };
  const float m = ld(g1_body_mass + b);
  float u1[3], u2[3], u3[3], FA[3], FB[3], Iom[3], Ial[3], NA[3], NBc[3], t[3];
  cross(alA, c, u1);
  cross(om, c, u2);
  cross(om, u2, u3);
  for (int k = 0; k < 3; k++) FA[k] = m * (aoA[k] + u1[k] + u3[k]);
  Iv(om, Iom);
  Iv(alA, Ial);
  cross(om, Iom, t);
  for (int k = 0; k < 3; k++) NA[k] = Ial[k] + t[k];
  cross(alB, c, u1);
  for (int k = 0; k < 3; k++) FB[k] = m * (aoB[k] + u1[k]);
  Iv(alB, NBc);
  for (int k = 0; k < 3; k++) {
    J.cw[k] = cw[k]; J.c[k] = c[k]; J.FA[k] = FA[k]; J.Iom[k] = Iom[k]; J.Ial[k] = Ial[k]; J.om[k] = om[k];
    J.alA[k] = alA[k]; J.alB[k] = alB[k]; J.FB[k] = FB[k]; J.NBc[k] = NBc[k]; J.X[k] = X[k];
  }
  J.I[0] = I[0][0]; J.I[1] = I[1][1]; J.I[2] = I[2][2]; J.I[3] = I[0][1]; J.I[4] = I[0][2]; J.I[5] = I[1][2];
  J.c[3] = m;
  // the own wrenches at the origin (N + cw x F, F) of both channels; G(lambda) comes in step 4
  cross(cw, FA, t);
  for (int k = 0; k < 3; k++) { J.SWA[k] = NA[k] + t[k]; J.SWA[3 + k] = FA[k]; }
  cross(cw, FB, t);
  for (int k = 0; k < 3; k++) { J.SWB[k] = NBc[k] + t[k]; J.SWB[3 + k] = FB[k]; }
  for (int k = 0; k < 6; k++) J.SGL[k] = 0.f;
  if (b >= 2) {
    const int p = ldi(g1_body_parent + b);
    for (int k = 0; k < 3; k++) { J.w[k] = W.ax[b + 4][k]; J.r[k] = X[k] - s.X[p][k]; }
  } else {
    for (int k = 0; k < 3; k++) { J.w[k] = 0.f; J.r[k] = 0.f; }
  }
}

// thread i < NV: dof i's motion vector s_i = (w, X x w) (root translations: (0, e_i); root rotations: the pelvis's
// axes about its origin; hinges: the axis through the body's origin)
__device__ __forceinline__ void jac_prep_dof_motion(JRec& R, const AWorld& s, const AdjShared& W, int i) {
  if (i < 3) {
    for (int k = 0; k < 6; k++) R.S6[i][k] = k == 3 + i ? 1.f : 0.f;
    return;
  }
  const int b = i < 6 ? 1 : i - 4;
  float xw[3];
  cross(s.X[b], W.ax[i], xw);
  for (int k = 0; k < 3; k++) { R.S6[i][k] = W.ax[i][k]; R.S6[i][3 + k] = xw[k]; }
}

// one warp, lane = body: G(lambda) onto the bodies (+ on body 2, - on body 1), then the subtree sums of SWA, SWB,
// SGL, level by level from the leaves
__device__ __forceinline__ void jac_prep_sums(JRec& R, int lane) {
  const int b = lane;
  if (b >= 1 && b < NB) {
    JBody& J = R.body[b];
    for (int q = R.cfirst[b]; q < R.cfirst[b + 1]; q++) {
      const JCon& C = R.con[R.cmem[q]];
      const float sg = C.b2 == b ? 1.f : -1.f;
      for (int k = 0; k < 6; k++) J.SGL[k] += sg * C.GL[k];
    }
  }
  __syncwarp();
  const int depth = b < NB ? ldi(g1_body_depth + b) : -1, nch = b < NB ? ldi(g1_body_nchild + b) : 0;
  for (int L = MAXD - 1; L >= 1; L--) {
    if (depth == L) {
      JBody& J = R.body[b];
      for (int ci = 0; ci < nch; ci++) {
        const JBody& C = R.body[ldi(g1_body_child + 3 * b + ci)];
        for (int k = 0; k < 6; k++) { J.SWA[k] += C.SWA[k]; J.SWB[k] += C.SWB[k]; J.SGL[k] += C.SGL[k]; }
      }
    }
    __syncwarp();
  }
}

// the whole preparation of record rec (every thread of the block)
__device__ __forceinline__ void jac_prep(JBlock& B, const float* rec, bool full, const float* fric_w,
                                         const float* com_w, const float* ctrl_w, float clamp_soft, int clamp_kv,
                                         int normal, int t) {
  JRec& R = B.R;
  AWorld& s = B.prep.s;
  AdjShared& W = B.prep.W;
  const int warp = t >> 5, lane = t & 31;
  jac_prep_state(B, rec, full, fric_w, com_w, ctrl_w, t);
  __syncthreads();
  if (warp == 0) adj_replay_kin(s, W, lane);
  else if (warp == 1) jac_prep_dofs(R, s, W, clamp_soft, clamp_kv, lane);
  else {
    jac_prep_lists(R, s, lane);
    adj_replay_rows(s, W, lane);
  }
  __syncthreads();
  if (warp == 0) {
    adj_replay_geoms(s, W, lane);
    jac_prep_dof_motion(R, s, W, lane);
    if (lane < NV - 32) jac_prep_dof_motion(R, s, W, 32 + lane);
  } else if (warp == 1) {
    adj_motion(s, W, s.qacc, W.VA, lane);
    if (lane >= 1 && lane < NB) jac_prep_body(R, s, W, lane);
  } else {
    adj_motion(s, W, s.qvel, W.VV, lane);
    if (!full) adj_mass_factor(s, W, B.prep.M, B.prep.Ic, R.LQ, R.dinvQ, lane);
  }
  __syncthreads();
  for (int i = t; i < 3 * R.ncon; i += JTHREADS) jac_prep_contact(R, s, W, normal, i);
  __syncthreads();
  if (warp == 0) jac_prep_sums(R, lane);
  __syncthreads();
}

// ---- one right-hand side through one record (the lane's column x: row r at x[r * JS]) -----------------------------
#define JX(o, i) x[((o) + (i)) * JS]

// Rows i0 .. i0 + NBK - 1 of the solve L v = b with a dense packed factor, in rows o.. of the lane's column: the NBK
// dot products over the entries q < i0 share each x[q] load (NBK independent chains), then the block's own triangle.
// Each row takes the same terms in the same order as a row-at-a-time solve.
template <int NBK>
__device__ __forceinline__ void jac_fwd_block(const float* L, const float* dinv, float* x, int o, int i0, int qs = 0) {
  float v[NBK];
  const float* Lr[NBK];
#pragma unroll
  for (int k = 0; k < NBK; k++) { v[k] = JX(o, i0 + k); Lr[k] = L + TRI(i0 + k, 0); }
#pragma unroll 2
  for (int q = qs; q < i0; q++) {
    const float xq = JX(o, q);
#pragma unroll
    for (int k = 0; k < NBK; k++) v[k] -= Lr[k][q] * xq;
  }
#pragma unroll
  for (int k = 0; k < NBK; k++) {
#pragma unroll
    for (int m = 0; m < k; m++) v[k] -= Lr[k][i0 + m] * v[m];
    v[k] *= dinv[i0 + k];
    JX(o, i0 + k) = v[k];
  }
}
// Rows i0 + NBK - 1 .. i0 of the solve L' v = b: the entries q >= i0 + NBK first (each x[q] load shared by the NBK
// rows; L(q, i0 .. i0 + NBK - 1) are consecutive in the packed row q), then the block's own triangle
template <int NBK>
__device__ __forceinline__ void jac_bwd_block(const float* L, const float* dinv, float* x, int o, int i0, int ce = NV,
                                              int js = NV) {
  float v[NBK];
#pragma unroll
  for (int k = 0; k < NBK; k++) v[k] = JX(o, i0 + k);
  int e = TRI(i0 + NBK, i0);
#pragma unroll 2
  for (int q = i0 + NBK; q < ce; q++) {
    const float xq = JX(o, q);
#pragma unroll
    for (int k = 0; k < NBK; k++) v[k] -= L[e + k] * xq;
    e += q + 1;
  }
  e = TRI(js, i0);
#pragma unroll 2
  for (int q = js; q < NV; q++) {
    const float xq = JX(o, q);
#pragma unroll
    for (int k = 0; k < NBK; k++) v[k] -= L[e + k] * xq;
    e += q + 1;
  }
#pragma unroll
  for (int k = NBK - 1; k >= 0; k--) {
#pragma unroll
    for (int m = NBK - 1; m > k; m--) v[k] -= L[TRI(i0 + m, i0 + k)] * v[m];
    v[k] *= dinv[i0 + k];
    JX(o, i0 + k) = v[k];
  }
}
// L_H in blocks of JBK rows, L_Q one block per segment of its order (at most 7 rows). Measured at B = 4096 on
// configuration-4 states, kernel alone: row at a time 6.25 ms; blocks of 4 / 4: 5.39; 8 / 8: 5.26; 8 / 4: 5.45;
// 5 / 7: 5.30; 7 / 7: 5.26; 6 / 7: 5.21 ms.
constexpr int JBK = 6, JBK_TAIL = NV % JBK, JBK_FULL = NV - JBK_TAIL;
constexpr int JQBK = 7;
// one segment of N rows from p0 (the same pattern ranges), in blocks of JQBK rows from its first row
template <int N>
__device__ __forceinline__ void jac_fwd_seg(const float* L, const float* dinv, float* x, int o, int p0, int qs) {
  constexpr int F = N < JQBK ? N : JQBK;
  jac_fwd_block<F>(L, dinv, x, o, p0, qs);
  if constexpr (N > F) jac_fwd_seg<N - F>(L, dinv, x, o, p0 + F, qs);
}
template <int N>
__device__ __forceinline__ void jac_bwd_seg(const float* L, const float* dinv, float* x, int o, int p0, int ce, int js) {
  constexpr int F = N < JQBK ? N : JQBK;
  if constexpr (N > F) jac_bwd_seg<N - F>(L, dinv, x, o, p0 + F, ce, js);
  jac_bwd_block<F>(L, dinv, x, o, p0, ce, js);
}

// the integrator, y = (M + h kv)^-1 abar_adv, lambda = H^-1 abar*, and the limit rows' and actuators' terms
__device__ __forceinline__ void jac_rhs_solves(const JRec& R, float* x) {
  const float h = G1_TIMESTEP;
  // q' = q (+) h v', v' = v + h a_adv: the input velocity gets vbar'_tot = vbar' + h qbar' (translations, hinges;
  // the rotation: h J_r' qbar'_rot), the input tangent qbar' (the rotation: R(phi) qbar'_rot); abar_adv = h vbar'_tot
  const float tb[3] = {JX(JO_Q, 3), JX(JO_Q, 4), JX(JO_Q, 5)};
#pragma unroll 5
  for (int i = 0; i < NV; i++) {
    float vt = JX(JO_V, i), ql;
    if (i < 3 || i >= 6) {
      ql = JX(JO_Q, i);
      vt += h * ql;
    } else {
      const float* a1 = R.A1 + 3 * (i - 3);
      const float* a2 = R.A2 + 3 * (i - 3);
      vt += h * (a1[0] * tb[0] + a1[1] * tb[1] + a1[2] * tb[2]);
      ql = a2[0] * tb[0] + a2[1] * tb[1] + a2[2] * tb[2];
    }
    JX(JO_V, i) = vt;
    JX(JO_Q, i) = ql;
    JX(JO_LAM, i) = h * vt;
  }
  // y with L_Q (tree-block order): position p of the solve is dof tb_dof(p), worked on in the slot rows
#pragma unroll 5
  for (int p = 0; p < NV; p++) JX(JO_SLOT, p) = JX(JO_LAM, tb_dof(p));
  // L_Q's pattern in tree-block order, by segment (legs 0..5 and 6..11, arms 12..18 and 19..25, waist 26..28, root
  // 29..34): a row's entries left of the diagonal are q in [qs, p) (qs: its segment's first row; the waist's: 12, the
  // root's: 0); a column's entries below it are q in (p, ce) (ce: its segment's end; the waist's and root's: NV) and
  // [js, NV) (the legs': the root, 29; the arms': the waist and root, 26)
  const float* LQ = R.LQ;
  const float* dQ = R.dinvQ;
  jac_fwd_seg<6>(LQ, dQ, x, JO_SLOT, 0, 0);     // left leg
  jac_fwd_seg<6>(LQ, dQ, x, JO_SLOT, 6, 6);     // right leg
  jac_fwd_seg<7>(LQ, dQ, x, JO_SLOT, 12, 12);   // left arm
  jac_fwd_seg<7>(LQ, dQ, x, JO_SLOT, 19, 19);   // right arm
  jac_fwd_seg<3>(LQ, dQ, x, JO_SLOT, 26, 12);   // waist (below both arms)
  jac_fwd_seg<6>(LQ, dQ, x, JO_SLOT, 29, 0);    // root (below everything)
  jac_bwd_seg<6>(LQ, dQ, x, JO_SLOT, 29, NV, NV);
  jac_bwd_seg<3>(LQ, dQ, x, JO_SLOT, 26, NV, NV);
  jac_bwd_seg<7>(LQ, dQ, x, JO_SLOT, 19, 26, 26);
  jac_bwd_seg<7>(LQ, dQ, x, JO_SLOT, 12, 19, 26);
  jac_bwd_seg<6>(LQ, dQ, x, JO_SLOT, 6, 12, 29);
  jac_bwd_seg<6>(LQ, dQ, x, JO_SLOT, 0, 6, 29);
  // abar* = abar_adv - h kv y; lambda with L_H (dof order)
#pragma unroll 5
  for (int p = 0; p < NV; p++) {
    const int i = tb_dof(p);
    const float y = JX(JO_SLOT, p);
    JX(JO_Y, i) = y;
    JX(JO_LAM, i) -= h * ld(g1_dof_kv + i) * y;
  }
#pragma unroll 1
  for (int i0 = 0; i0 < JBK_FULL; i0 += JBK) jac_fwd_block<JBK>(R.LH, R.dinvH, x, JO_LAM, i0);
  if constexpr (JBK_TAIL > 0) {
    jac_fwd_block<JBK_TAIL>(R.LH, R.dinvH, x, JO_LAM, JBK_FULL);
    jac_bwd_block<JBK_TAIL>(R.LH, R.dinvH, x, JO_LAM, JBK_FULL);
  }
#pragma unroll 1
  for (int i0 = JBK_FULL - JBK; i0 >= 0; i0 -= JBK) jac_bwd_block<JBK>(R.LH, R.dinvH, x, JO_LAM, i0);
  // the limit rows and the actuators
#pragma unroll 5
  for (int i = 6; i < NV; i++) {
    const float lam = JX(JO_LAM, i);
    JX(JO_Q, i) += R.dcq[i] * lam;
    JX(JO_V, i) += R.dcv[i] * lam;
    JX(JO_U, i - 6) += R.dcu[i] * lam;
  }
}

// the motion of body b (angular, linear at the origin) of the generalised vector in rows o.. : its path's dofs
__device__ __forceinline__ void jac_path_motion(const JRec& R, const float* x, int o, int b, float* V) {
  for (int k = 0; k < 6; k++) V[k] = 0.f;
  for (int a = b; a >= 1; a = ldi(g1_body_parent + a)) {
    const int d0 = a >= 2 ? a + 4 : 0, d1 = a >= 2 ? a + 5 : 6;
    for (int d = d0; d < d1; d++) {
      const float v = JX(o, d);
      float s6[6];
      jv6(R.S6[d], s6);
      for (int k = 0; k < 6; k++) V[k] += s6[k] * v;
    }
  }
}

// lambda's relative motion V(b2) - V(b1) of a self contact from the dofs between the two bodies (their common
// ancestors' terms cancel and are left out): the same bits at both of the contact's bodies, so the two pose wrenches,
// which cancel under a motion of the pair as a whole, see the same dV
__device__ __forceinline__ void jac_rel_motion(const JRec& R, const float* x, int b1, int b2, float* dV) {
  for (int k = 0; k < 6; k++) dV[k] = 0.f;
  int a = b2, c = b1, da = ldi(g1_body_depth + a), dc = ldi(g1_body_depth + c);
  while (a != c) {
    const bool up2 = da >= dc;
    const int e = up2 ? a : c;
    const float sg = up2 ? 1.f : -1.f;
    const int d0 = e >= 2 ? e + 4 : 0, d1 = e >= 2 ? e + 5 : 6;
    for (int d = d0; d < d1; d++) {
      const float v = sg * JX(JO_LAM, d);
      float s6[6];
      jv6(R.S6[d], s6);
      for (int k = 0; k < 6; k++) dV[k] += s6[k] * v;
    }
    if (up2) { a = ldi(g1_body_parent + a); da--; } else { c = ldi(g1_body_parent + c); dc--; }
  }
}

__device__ __forceinline__ void sym_mul(const float* I, const float* v, float* o) {  // I: xx, yy, zz, xy, xz, yz
  o[0] = I[0] * v[0] + I[3] * v[1] + I[4] * v[2];
  o[1] = I[3] * v[0] + I[1] * v[1] + I[5] * v[2];
  o[2] = I[4] * v[0] + I[5] * v[1] + I[2] * v[2];
}

// a body's own terms of both ID channels for the motions VL (lambda, channel A: weight -1) and VY (y, channel B):
// the cotangents of its angular velocity and both channels' accelerations, its rotation (rho) and the pose wrench of
// its COM point (P)
__device__ __forceinline__ void jac_own(const JBody& J, const float* VL, const float* VY, float* omb, float* alAb,
                                        float* aoAb, float* alBb, float* aoBb, float* rho, float* P) {
  float cw[3], c[3], Iw[6], FA[3], Iom[3], Ial[3], om[3], alA[3], alB[3], FB[3], NBc[3];
  jv3(J.cw, cw); jv6(J.I, Iw); jv3(J.FA, FA); jv3(J.Iom, Iom); jv3(J.Ial, Ial); jv3(J.om, om); jv3(J.alA, alA);
  jv3(J.alB, alB); jv3(J.FB, FB); jv3(J.NBc, NBc);
  const float4 c4 = *reinterpret_cast<const float4*>(J.c);
  c[0] = c4.x; c[1] = c4.y; c[2] = c4.z;
  const float m = c4.w;
  float t[3], cwb[3];
  {  // channel A: psi_A = -<W_b, V^lambda_b>, W_b = (N + cw x F, F), F = m (ao + al x c + om x (om x c))
    float Fb[3], Nb[3], Inb[3], n2[3], In2[3], acb[3], cb[3], z[3], zb[3];
    cross(VL, cw, t);
    for (int k = 0; k < 3; k++) { Fb[k] = -(VL[3 + k] + t[k]); Nb[k] = -VL[k]; }
    cross(VL, FA, cwb);
    sym_mul(Iw, Nb, Inb);
    for (int k = 0; k < 3; k++) alAb[k] = Inb[k];
    cross(Nb, om, n2);
    sym_mul(Iw, n2, In2);
    cross(Iom, Nb, t);
    for (int k = 0; k < 3; k++) omb[k] = t[k] + In2[k];
    cross(Ial, Nb, rho);
    cross(Inb, alA, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
    cross(Iom, n2, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
    cross(In2, om, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
    for (int k = 0; k < 3; k++) { acb[k] = m * Fb[k]; aoAb[k] = acb[k]; }
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
    cross(c, cb, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
  }
  {  // channel B: weight +1, om = 0
    float Fb[3], Inb[3], acb[3], cb[3];
    cross(VY, cw, t);
    for (int k = 0; k < 3; k++) Fb[k] = VY[3 + k] + t[k];
    cross(FB, VY, t);
    for (int k = 0; k < 3; k++) cwb[k] += t[k];
    sym_mul(Iw, VY, Inb);
    for (int k = 0; k < 3; k++) alBb[k] = Inb[k];
    cross(NBc, VY, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
    cross(Inb, alB, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
    for (int k = 0; k < 3; k++) { acb[k] = m * Fb[k]; aoBb[k] = acb[k]; }
    cross(c, acb, t);
    for (int k = 0; k < 3; k++) alBb[k] += t[k];
    cross(acb, alB, cb);
    cross(c, cb, t);
    for (int k = 0; k < 3; k++) rho[k] += t[k];
  }
  cross(cw, cwb, t);  // the COM point's cotangent: a force at cw
  for (int k = 0; k < 3; k++) { P[k] = t[k]; P[3 + k] = cwb[k]; }
}

// the hand-over of a child to its parent b (h: the recursion's cotangents omb, alAb, aoAb, alBb, aoBb, the
// relative-position force rb, then the subtree sums of G(a*), G(v) and the pose wrenches)
__device__ __forceinline__ void jac_inflow(const float* hv, const float* X, float* omb, float* alAb, float* aoAb,
                                           float* alBb, float* aoBb, float* P, float* SGa, float* SGv, float* SP) {
  for (int k = 0; k < 3; k++) {
    omb[k] += hv[k]; alAb[k] += hv[3 + k]; aoAb[k] += hv[6 + k]; alBb[k] += hv[9 + k]; aoBb[k] += hv[12 + k];
  }
  float t[3];
  cross(X, hv + 15, t);  // the child's rbar: force -rbar at this body's origin
  for (int k = 0; k < 3; k++) { P[k] -= t[k]; P[3 + k] -= hv[15 + k]; }
  for (int k = 0; k < 6; k++) { SGa[k] += hv[18 + k]; SGv[k] += hv[24 + k]; SP[k] += hv[30 + k]; }
}

// the leaf-to-root pass (as adj_sweep, one cotangent per lane): bodies NB - 1 .. 1
__device__ __forceinline__ void jac_rhs_sweep(const JRec& R, float* x) {
  float VL[6], VY[6], hv[JSLOT];
  int parked = -1;  // the body whose hand-over is parked in the slot rows
#pragma unroll 1
  for (int b = NB - 1; b >= 1; b--) {
    const JBody& J = R.body[b];
    float Xb[3];
    jv3(J.X, Xb);
    const bool carried = b + 1 < NB && ldi(g1_body_parent + b + 1) == b;  // hv is the child b + 1's hand-over
    if (carried) {
      const int dc = b + 5;  // the child's hinge
      const float xl = JX(JO_LAM, dc), xy = JX(JO_Y, dc);
      float s6[6];
      jv6(R.S6[dc], s6);
      for (int k = 0; k < 6; k++) { VL[k] -= s6[k] * xl; VY[k] -= s6[k] * xy; }
    } else {
      jac_path_motion(R, x, JO_LAM, b, VL);
      jac_path_motion(R, x, JO_Y, b, VY);
    }
    float omb[3], alAb[3], aoAb[3], alBb[3], aoBb[3], rho[3], P[6], SGa[6], SGv[6], SP[6];
    jac_own(J, VL, VY, omb, alAb, aoAb, alBb, aoBb, rho, P);
    for (int k = 0; k < 6; k++) { SGa[k] = 0.f; SGv[k] = 0.f; SP[k] = 0.f; }
    // the contacts at this body: G(a*), G(v) (+ on body 2, - on body 1) and this body's pose wrench
#pragma unroll 1
    for (int q = R.cfirst[b]; q < R.cfirst[b + 1]; q++) {
      const JCon& C = R.con[R.cmem[q]];
      const bool two = C.b2 == b;
      float dV[6];
      if (C.b1 >= 1) jac_rel_motion(R, x, C.b1, C.b2, dV);
      else for (int k = 0; k < 6; k++) dV[k] = VL[k];  // (the world: a plane, body 2 only)
      const float* Mp = two ? C.P2 : C.P1;
      const float sg = two ? 1.f : -1.f;
#pragma unroll
      for (int r = 0; r < 6; r++) {
        float g = 0.f, pw = 0.f;
#pragma unroll
        for (int k = 0; k < 6; k++) { g += C.Ga[6 * r + k] * dV[k]; pw += Mp[6 * r + k] * dV[k]; }
        SGa[r] += sg * g;
        SGv[r] += sg * (C.bb * g);
        P[r] += pw;
      }
    }
    if (carried) jac_inflow(hv, Xb, omb, alAb, aoAb, alBb, aoBb, P, SGa, SGv, SP);
    if (parked == b) {
      float sv[JSLOT];
      for (int k = 0; k < JSLOT; k++) sv[k] = JX(JO_SLOT, k);
      jac_inflow(sv, Xb, omb, alAb, aoAb, alBb, aoBb, P, SGa, SGv, SP);
      parked = -1;
    }
    float t[3];
    if (b >= 2) {
      const int d = b + 4, p = ldi(g1_body_parent + b);
      const JBody& Pp = R.body[p];
      float wj[3], rj[3], pom[3], palA[3], palB[3];
      jv3(J.w, wj); jv3(J.r, rj); jv3(Pp.om, pom); jv3(Pp.alA, palA); jv3(Pp.alB, palB);
      const float vd = R.vd[d], ad = R.ad[d], xd = R.xd[d];
      float wb[3], z[3], zb[3], rb[3], aw[3], wv[3];
      // channel A: om_b = om_p + w vd; al_b = al_p + om_p x (w vd) + w ad; ao_b = ao_p + al_p x r + om_p x (om_p x r)
      for (int k = 0; k < 3; k++) {
        hv[k] = omb[k]; hv[3 + k] = alAb[k]; hv[6 + k] = aoAb[k];
        wb[k] = vd * omb[k] + ad * alAb[k];
        wv[k] = wj[k] * vd;
      }
      float vbar = dot3(wj, omb);
      cross(wv, alAb, t);
      for (int k = 0; k < 3; k++) hv[k] += t[k];
      cross(alAb, pom, aw);
      for (int k = 0; k < 3; k++) wb[k] += vd * aw[k];
      vbar += dot3(wj, aw);
      cross(rj, aoAb, t);
      for (int k = 0; k < 3; k++) hv[3 + k] += t[k];
      cross(pom, rj, z);
      cross(aoAb, pom, zb);
      cross(z, aoAb, t);
      for (int k = 0; k < 3; k++) hv[k] += t[k];
      cross(rj, zb, t);
      for (int k = 0; k < 3; k++) hv[k] += t[k];
      cross(aoAb, palA, rb);
      cross(zb, pom, t);
      for (int k = 0; k < 3; k++) rb[k] += t[k];
      // channel B: al_b = al_p + w xd; ao_b = ao_p + al_p x r
      for (int k = 0; k < 3; k++) { hv[9 + k] = alBb[k]; hv[12 + k] = aoBb[k]; wb[k] += xd * alBb[k]; }
      cross(rj, aoBb, t);
      for (int k = 0; k < 3; k++) hv[9 + k] += t[k];
      cross(aoBb, palB, t);
      for (int k = 0; k < 3; k++) rb[k] += t[k];
      // r = X - Xp: force rbar at X (this body), -rbar at Xp (the parent)
      cross(Xb, rb, t);
      for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += rb[k]; hv[15 + k] = rb[k]; }
      // the dof's motion vector s = (w, X x w): sbar = -lam W_A + y W_B + lam G_l + a G_a + v G_v (subtree sums)
      const float lam = JX(JO_LAM, d), yd = JX(JO_Y, d);
      float sb[6], swa[6], swb[6], sgl[6];
      jv6(J.SWA, swa); jv6(J.SWB, swb); jv6(J.SGL, sgl);
      for (int k = 0; k < 6; k++)
        sb[k] = -lam * swa[k] + yd * swb[k] + lam * sgl[k] + ad * SGa[k] + vd * SGv[k];
      JX(JO_V, d) += vbar + wrench_dot(SGv, wj, Xb);
      cross(sb + 3, Xb, t);
      for (int k = 0; k < 3; k++) wb[k] += sb[k] + t[k];
      float xf[3];
      cross(wj, sb + 3, xf);
      cross(Xb, xf, t);
      for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += xf[k]; }
      cross(wj, wb, t);  // the axis rotates with the body
      for (int k = 0; k < 3; k++) rho[k] += t[k];
      for (int k = 0; k < 3; k++) P[k] += rho[k];
      for (int k = 0; k < 6; k++) SP[k] += P[k];
      JX(JO_Q, d) += wrench_dot(SP, wj, Xb);
      for (int k = 0; k < 6; k++) { hv[18 + k] = SGa[k]; hv[24 + k] = SGv[k]; hv[30 + k] = SP[k]; }
      if (p != b - 1) {  // the parent is not visited next: park the hand-over (added to one parked for p)
        const bool add = parked == p;
        for (int k = 0; k < JSLOT; k++) JX(JO_SLOT, k) = add ? JX(JO_SLOT, k) + hv[k] : hv[k];
        parked = p;
      }
    } else {  // the root: its 6 dofs; om_1 = sum_i w_i v_i, al_1 = sum_i w_i a_i (w_i: the pelvis's axes)
      float wbr[3][3];
      for (int i = 0; i < 3; i++) {
        const float* w = R.S6[3 + i];
        JX(JO_V, 3 + i) += dot3(w, omb);
        for (int k = 0; k < 3; k++)
          wbr[i][k] = R.vd[3 + i] * omb[k] + R.ad[3 + i] * alAb[k] + R.xd[3 + i] * alBb[k];
      }
      float swa[6], swb[6], sgl[6];
      jv6(J.SWA, swa); jv6(J.SWB, swb); jv6(J.SGL, sgl);
      for (int i = 0; i < 6; i++) {
        const float lam = JX(JO_LAM, i), yd = JX(JO_Y, i);
        float sb[6];
        for (int k = 0; k < 6; k++)
          sb[k] = -lam * swa[k] + yd * swb[k] + lam * sgl[k] + R.ad[i] * SGa[k] + R.vd[i] * SGv[k];
        if (i < 3) {
          JX(JO_V, i) += SGv[3 + i];  // s = (0, e_i)
        } else {
          const float* w = R.S6[i];
          JX(JO_V, i) += wrench_dot(SGv, w, Xb);
          cross(sb + 3, Xb, t);
          for (int k = 0; k < 3; k++) wbr[i - 3][k] += sb[k] + t[k];
          float xf[3];
          cross(w, sb + 3, xf);
          cross(Xb, xf, t);
          for (int k = 0; k < 3; k++) { P[k] += t[k]; P[3 + k] += xf[k]; }
        }
      }
      for (int i = 0; i < 3; i++) {
        cross(R.S6[3 + i], wbr[i], t);
        for (int k = 0; k < 3; k++) rho[k] += t[k];
      }
      for (int k = 0; k < 3; k++) P[k] += rho[k];
      for (int k = 0; k < 6; k++) SP[k] += P[k];
      for (int i = 0; i < 3; i++) JX(JO_Q, i) += SP[3 + i];
      for (int i = 3; i < 6; i++) JX(JO_Q, i) += wrench_dot(SP, R.S6[i], Xb);
    }
  }
}

}  // namespace nbg1
