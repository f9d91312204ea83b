// Kinematics outputs of a state and their VJP (one warp per world, lane b = body b, the tree one depth level at a
// time). Outputs, as the reference's `kinematics=True` (src/nablaengine/g1_engine/kinematics.py:1-47, MuJoCo MJX's
// kinematics + com_pos + com_vel):
//   qpos_n (NQ)       qpos with the root quaternion normalised;
//   xpos (NB,3), xquat (NB,4)  the body frames (the world body: 0, (1,0,0,0)); a hinge body: xpos[p] + R_p body_pos,
//                     xquat[p] body_quat axis_angle(axis, q) (products, not renormalised);
//   subtree_com (NB,3)  sum(m xipos) / sum(m) per subtree (the torso's ipos plus the per-world com offset);
//                     subtree_com[0] = subtree_com[1];
//   cvel (NB,6)       [W_b; V_b + W_b x (subtree_com[1] - xpos[b])]: W_b the world angular velocity, V_b the velocity
//                     of the body origin (root: R_1 qvel[3:6], qvel[0:3]; child: W_p + a_b qd_b, V_p + W_p x (X_b -
//                     X_p)); body 0 zeros.
// The VJP recomputes the state and reverses it: cvel's cotangents into the twists' (W bar, V bar) and the reference
// point's (a force on every subtree COM), the subtree COMs' into forces at each body's COM (a root-to-leaf sum of the
// subtree sums' cotangents), the poses' into forces and torques per body; the twist recursion leaf to root (qvel's
// cotangents, and the recursion's own pose dependence: the lever arms X_c - X_b and the rotating hinge axes); then
// the pose cotangents as wrenches about the world origin summed over subtrees, projected on each dof's motion: the
// hinge angles, the root translation, and the root quaternion through its normalisation.
#pragma once
#include "nb_g1_step.cuh"

namespace nbg1 {

constexpr int KWPB = 4;  // worlds (warps) per block of the kinematics kernels

struct KinS {  // one world's kinematics state and its VJP accumulators (4.7 KB)
  float Q[NB][4], X[NB][3], W[NB][3], V[NB][3], C[NB][3], Mt[NB], xi[NB][3];
  float qpos[NQ], qvel[NV], com[3], qn_norm;
  float bW[NB][3], bV[NB][3];    // twist cotangents (own, then the pushes to the parent: pW, pV)
  float pW[NB][3], pV[NB][3], rb[NB][3];
  float Fo[NB][6];               // per body: moment about the world origin, force (pose cotangents), then subtree sums
  float G[NB][3];                // root-to-body sums of the subtree sums' cotangents
};

__device__ __forceinline__ void kin_ipos(int b, const float* com, float* ip) {
  for (int k = 0; k < 3; k++) ip[k] = ld(g1_body_ipos + 3 * b + k) + (b == G1_TORSO ? com[k] : 0.f);
}

// poses, twists, COM points, subtree COMs (C) and masses (Mt) of the state in s.qpos / s.qvel / s.com
__device__ __noinline__ void kin_state(KinS& s, int lane) {
  const int b = lane, depth = b < NB ? ldi(g1_body_depth + b) : -1;
  if (lane == 0) {
    s.Q[0][0] = 1.f; s.Q[0][1] = s.Q[0][2] = s.Q[0][3] = 0.f;
    for (int k = 0; k < 3; k++) s.X[0][k] = s.W[0][k] = s.V[0][k] = 0.f;
  }
  __syncwarp();
  for (int L = 1; L <= MAXD; L++) {
    if (depth == L) {
      if (b == 1) {
        const float q[4] = {s.qpos[3], s.qpos[4], s.qpos[5], s.qpos[6]};
        const float n = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
        for (int k = 0; k < 4; k++) s.Q[1][k] = q[k] / n;
        s.qn_norm = n;
        const float wl[3] = {s.qvel[3], s.qvel[4], s.qvel[5]};
        float w[3];
        qrot(s.Q[1], wl, w);
        for (int k = 0; k < 3; k++) { s.X[1][k] = s.qpos[k]; s.W[1][k] = w[k]; s.V[1][k] = s.qvel[k]; }
      } else {
        const int p = ldi(g1_body_parent + b), d = b + 4;
        const float bq[4] = {ld(g1_body_quat + 4 * b), ld(g1_body_quat + 4 * b + 1), ld(g1_body_quat + 4 * b + 2),
                             ld(g1_body_quat + 4 * b + 3)};
        const float bp[3] = {ld(g1_body_pos + 3 * b), ld(g1_body_pos + 3 * b + 1), ld(g1_body_pos + 3 * b + 2)};
        const float ax[3] = {ld(g1_body_axis + 3 * b), ld(g1_body_axis + 3 * b + 1), ld(g1_body_axis + 3 * b + 2)};
        float q0[4], t[3], Q[4], aw[3], sn, cs, u[3];
        qmul(s.Q[p], bq, q0);
        qrot(s.Q[p], bp, t);
        sincosf(0.5f * s.qpos[d + 1], &sn, &cs);
        const float ha[4] = {cs, sn * ax[0], sn * ax[1], sn * ax[2]};
        qmul(q0, ha, Q);
        qrot(Q, ax, aw);
        float X[3], r[3];
        for (int k = 0; k < 3; k++) { X[k] = s.X[p][k] + t[k]; r[k] = X[k] - s.X[p][k]; }
        cross(s.W[p], r, u);
        const float qd = s.qvel[d];
        for (int k = 0; k < 4; k++) s.Q[b][k] = Q[k];
        for (int k = 0; k < 3; k++) {
          s.X[b][k] = X[k];
          s.W[b][k] = s.W[p][k] + aw[k] * qd;
          s.V[b][k] = s.V[p][k] + u[k];
        }
      }
    }
    __syncwarp();
  }
  // COM points and subtree sums (leaf to root, children pulled)
  float S[3] = {0.f, 0.f, 0.f}, m = 0.f;
  if (b >= 1 && b < NB) {
    float ip[3], c[3];
    kin_ipos(b, s.com, ip);
    qrot(s.Q[b], ip, c);
    m = ld(g1_body_mass + b);
    for (int k = 0; k < 3; k++) { s.xi[b][k] = s.X[b][k] + c[k]; S[k] = m * s.xi[b][k]; s.C[b][k] = S[k]; }
    s.Mt[b] = m;
  }
  __syncwarp();
  const int nch = b >= 1 && b < NB ? ldi(g1_body_nchild + b) : 0;
  for (int L = MAXD - 1; L >= 1; L--) {
    if (depth == L && nch > 0) {
      for (int i = 0; i < nch; i++) {
        const int c = ldi(g1_body_child + 3 * b + i);
        for (int k = 0; k < 3; k++) S[k] += s.C[c][k];
        m += s.Mt[c];
      }
      for (int k = 0; k < 3; k++) s.C[b][k] = S[k];
      s.Mt[b] = m;
    }
    __syncwarp();
  }
  if (b >= 1 && b < NB)
    for (int k = 0; k < 3; k++) s.C[b][k] = S[k] / m;
  __syncwarp();
  if (lane == 0) {
    for (int k = 0; k < 3; k++) s.C[0][k] = s.C[1][k];
    s.Mt[0] = s.Mt[1];
  }
  __syncwarp();
}

__device__ __forceinline__ void kin_load(KinS& s, size_t w, const float* qpos, const float* qvel, const float* com,
                                         int lane) {
  for (int i = lane; i < NQ; i += 32) s.qpos[i] = qpos[w * NQ + i];
  for (int i = lane; i < NV; i += 32) s.qvel[i] = qvel[w * NV + i];
  if (lane < 3) s.com[lane] = com[w * 3 + lane];
  __syncwarp();
}

__global__ void __launch_bounds__(KWPB * 32) k_kin(int nw, const float* __restrict__ qpos,
                                                   const float* __restrict__ qvel, const float* __restrict__ com,
                                                   float* __restrict__ qn, float* __restrict__ xpos,
                                                   float* __restrict__ xquat, float* __restrict__ cvel,
                                                   float* __restrict__ sc) {
  __shared__ KinS sm[KWPB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * KWPB + warp;
  if (w >= nw) return;  // whole warps
  KinS& s = sm[warp];
  const size_t w64 = (size_t)w;
  kin_load(s, w64, qpos, qvel, com, lane);
  kin_state(s, lane);
  for (int i = lane; i < NQ; i += 32) qn[w64 * NQ + i] = i >= 3 && i < 7 ? s.Q[1][i - 3] : s.qpos[i];
  for (int i = lane; i < NB * 3; i += 32) {
    xpos[w64 * NB * 3 + i] = (&s.X[0][0])[i];
    sc[w64 * NB * 3 + i] = (&s.C[0][0])[i];
  }
  for (int i = lane; i < NB * 4; i += 32) xquat[w64 * NB * 4 + i] = (&s.Q[0][0])[i];
  const int b = lane;
  if (b < NB) {
    float o[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (b >= 1) {
      float r[3], u[3];
      for (int k = 0; k < 3; k++) r[k] = s.C[1][k] - s.X[b][k];
      cross(s.W[b], r, u);
      for (int k = 0; k < 3; k++) { o[k] = s.W[b][k]; o[3 + k] = s.V[b][k] + u[k]; }
    }
    for (int k = 0; k < 6; k++) cvel[(w64 * NB + b) * 6 + k] = o[k];
  }
}

// adds force f at point p to the (moment about the origin, force) accumulator F
__device__ __forceinline__ void add_force(float* F, const float* p, const float* f) {
  float t[3];
  cross(p, f, t);
  for (int k = 0; k < 3; k++) { F[k] += t[k]; F[3 + k] += f[k]; }
}

__global__ void __launch_bounds__(KWPB * 32) k_kin_vjp(int nw, const float* __restrict__ qpos,
                                                       const float* __restrict__ qvel, const float* __restrict__ com,
                                                       const float* __restrict__ gqn, const float* __restrict__ gxpos,
                                                       const float* __restrict__ gxquat,
                                                       const float* __restrict__ gcvel, const float* __restrict__ gsc,
                                                       const float* __restrict__ gq_in,
                                                       const float* __restrict__ gv_in, float* __restrict__ gq,
                                                       float* __restrict__ gv) {
  __shared__ KinS sm[KWPB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * KWPB + warp;
  if (w >= nw) return;
  KinS& s = sm[warp];
  const size_t w64 = (size_t)w;
  kin_load(s, w64, qpos, qvel, com, lane);
  kin_state(s, lane);
  const int b = lane, depth = b < NB ? ldi(g1_body_depth + b) : -1;
  const bool body = b >= 1 && b < NB;
  const size_t row = w64 * NB + (b < NB ? b : 0);
  // per body: cvel -> twist cotangents and the reference point; xpos, xquat -> force and torque
  float F[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, c1b[3] = {0.f, 0.f, 0.f};
  if (body) {
    float wb[3], ub[3], r[3], t[3];
    for (int k = 0; k < 3; k++) {
      wb[k] = gcvel[row * 6 + k]; ub[k] = gcvel[row * 6 + 3 + k]; r[k] = s.C[1][k] - s.X[b][k];
    }
    cross(r, ub, t);  // W bar += r x ubar
    for (int k = 0; k < 3; k++) { s.bW[b][k] = wb[k] + t[k]; s.bV[b][k] = ub[k]; }
    cross(ub, s.W[b], c1b);  // rbar = ubar x W: the reference point C_1 gets it, X_b minus it
    float f[3];
    for (int k = 0; k < 3; k++) f[k] = gxpos[row * 3 + k] - c1b[k];
    add_force(F, s.X[b], f);
    if (b >= 2) {  // the frame's rotation: tau = 1/2 vec(g Q*)
      const float g[4] = {gxquat[row * 4], gxquat[row * 4 + 1], gxquat[row * 4 + 2], gxquat[row * 4 + 3]};
      const float qc[4] = {s.Q[b][0], -s.Q[b][1], -s.Q[b][2], -s.Q[b][3]};
      float o[4];
      qmul(g, qc, o);
      for (int k = 0; k < 3; k++) F[k] += 0.5f * o[1 + k];
    }
  }
  // the subtree COMs' cotangents: C_b = S_b / M_b; C_1 also gets subtree_com[0]'s and every cvel's reference point
  float sb[3] = {0.f, 0.f, 0.f};
  for (int k = 0; k < 3; k++) c1b[k] = warp_sum(c1b[k]);
  if (body) {
    for (int k = 0; k < 3; k++) {
      float g = gsc[row * 3 + k];
      if (b == 1) g += gsc[w64 * NB * 3 + k] + c1b[k];
      sb[k] = g / s.Mt[b];
    }
  }
  // root-to-body sums G_b = sum of S bar over the path 1 .. b; the COM point xi_b then carries the force m_b G_b
  if (lane == 1)
    for (int k = 0; k < 3; k++) s.G[1][k] = sb[k];
  __syncwarp();
  for (int L = 2; L <= MAXD; L++) {
    if (depth == L) {
      const int p = ldi(g1_body_parent + b);
      for (int k = 0; k < 3; k++) s.G[b][k] = s.G[p][k] + sb[k];
    }
    __syncwarp();
  }
  if (body) {
    const float m = ld(g1_body_mass + b);
    const float f[3] = {m * s.G[b][0], m * s.G[b][1], m * s.G[b][2]};
    add_force(F, s.xi[b], f);
  }
  // the twist recursion, leaf to root: pull the children's pushes, then push to the parent
  const int nch = body ? ldi(g1_body_nchild + b) : 0;
  float gvd = 0.f;  // this body's hinge rate cotangent
  for (int L = MAXD; L >= 1; L--) {
    if (depth == L) {
      float Wb[3] = {s.bW[b][0], s.bW[b][1], s.bW[b][2]}, Vb[3] = {s.bV[b][0], s.bV[b][1], s.bV[b][2]};
      for (int i = 0; i < nch; i++) {
        const int c = ldi(g1_body_child + 3 * b + i);
        for (int k = 0; k < 3; k++) { Wb[k] += s.pW[c][k]; Vb[k] += s.pV[c][k]; }
        // the child's lever arm r_c = X_c - X_b: -rbar_c at this body's origin
        const float nr[3] = {-s.rb[c][0], -s.rb[c][1], -s.rb[c][2]};
        add_force(F, s.X[b], nr);
      }
      if (b >= 2) {
        const int p = ldi(g1_body_parent + b), d = b + 4;
        const float ax[3] = {ld(g1_body_axis + 3 * b), ld(g1_body_axis + 3 * b + 1), ld(g1_body_axis + 3 * b + 2)};
        float aw[3], r[3], t[3], rbar[3];
        qrot(s.Q[b], ax, aw);
        gvd = dot3(aw, Wb);
        const float qd = s.qvel[d];
        const float wq[3] = {qd * Wb[0], qd * Wb[1], qd * Wb[2]};
        cross(aw, wq, t);  // the hinge axis turns with the body
        for (int k = 0; k < 3; k++) { F[k] += t[k]; r[k] = s.X[b][k] - s.X[p][k]; }
        cross(r, Vb, t);
        cross(Vb, s.W[p], rbar);
        add_force(F, s.X[b], rbar);
        for (int k = 0; k < 3; k++) { s.pW[b][k] = Wb[k] + t[k]; s.pV[b][k] = Vb[k]; s.rb[b][k] = rbar[k]; }
      } else if (b == 1) {
        // W_1 = R w_local: w_local bar = R' W bar; the rotation: torque W_1 x W bar
        float t[3];
        cross(s.W[1], Wb, t);
        for (int k = 0; k < 3; k++) { F[k] += t[k]; s.bV[1][k] = Vb[k]; s.bW[1][k] = Wb[k]; }
      }
    }
    __syncwarp();
  }
  // subtree sums of the pose wrenches (leaf to root)
  for (int L = MAXD; L >= 1; L--) {
    if (depth == L) {
      for (int i = 0; i < nch; i++) {
        const int c = ldi(g1_body_child + 3 * b + i);
        for (int k = 0; k < 6; k++) F[k] += s.Fo[c][k];
      }
      for (int k = 0; k < 6; k++) s.Fo[b][k] = F[k];
    }
    __syncwarp();
  }
  float* oq = gq + w64 * NQ;
  float* ov = gv + w64 * NV;
  if (b >= 2 && b < NB) {  // hinge: the wrench on the motion (a, X_b x a), plus qpos_n's pass-through
    const int d = b + 4;
    const float ax[3] = {ld(g1_body_axis + 3 * b), ld(g1_body_axis + 3 * b + 1), ld(g1_body_axis + 3 * b + 2)};
    float aw[3], xa[3];
    qrot(s.Q[b], ax, aw);
    cross(s.X[b], aw, xa);
    const float g = dot3(F, aw) + dot3(F + 3, xa) + gqn[w64 * NQ + d + 1];
    oq[d + 1] = g + (gq_in ? gq_in[w64 * NQ + d + 1] : 0.f);
    ov[d] = gvd + (gv_in ? gv_in[w64 * NV + d] : 0.f);
  }
  if (lane == 1) {
    // root translation: the total force; root quaternion: the torque about the root origin, N = M_O - X_1 x F,
    // a = 2 (0, N) Q_1 + g_xquat[1] + g_qpos_n[3:7], through the normalisation: (a - u (u . a)) / |q|
    float N[3], t[3];
    cross(s.X[1], F + 3, t);
    for (int k = 0; k < 3; k++) N[k] = F[k] - t[k];
    const float n4[4] = {0.f, N[0], N[1], N[2]};
    float a[4];
    qmul(n4, s.Q[1], a);
    for (int k = 0; k < 4; k++)
      a[k] = 2.f * a[k] + gxquat[w64 * NB * 4 + 4 + k] + gqn[w64 * NQ + 3 + k];
    const float ua = s.Q[1][0] * a[0] + s.Q[1][1] * a[1] + s.Q[1][2] * a[2] + s.Q[1][3] * a[3];
    for (int k = 0; k < 4; k++)
      oq[3 + k] = (a[k] - s.Q[1][k] * ua) / s.qn_norm + (gq_in ? gq_in[w64 * NQ + 3 + k] : 0.f);
    for (int k = 0; k < 3; k++)
      oq[k] = F[3 + k] + gqn[w64 * NQ + k] + (gq_in ? gq_in[w64 * NQ + k] : 0.f);
    // root velocities: V_1 = qvel[0:3], W_1 = R qvel[3:6]
    const float qc[4] = {s.Q[1][0], -s.Q[1][1], -s.Q[1][2], -s.Q[1][3]};
    float wl[3];
    qrot(qc, s.bW[1], wl);
    for (int k = 0; k < 3; k++) {
      ov[k] = s.bV[1][k] + (gv_in ? gv_in[w64 * NV + k] : 0.f);
      ov[3 + k] = wl[k] + (gv_in ? gv_in[w64 * NV + 3 + k] : 0.f);
    }
  }
}

}  // namespace nbg1
