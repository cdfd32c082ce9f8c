// C++ port of the reference's kernel test (cpp/src/tests.cpp:196-243,
// test_delta) against the C++ host API gdn::delta (gdn_delta.hpp): random
// seeded cases (B,L,H) with the reference's distributions, the kernel against
// the CPU oracle (oracle/gdn_oracle.c), max-relative error < 1e-5 on o,
// s_out and every collected state (the reference's bound is 2e-5).
// Built and run by tests/test_gpu_cpp.py; prints one "[ok]"/"[FAIL]" line
// per check and exits non-zero on any failure.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "gdn_delta.hpp"

extern "C" void oracle_recurrent(const float* q, const float* k, const float* v, const float* alpha,
                                 const float* beta, const float* S_in, float* S_out, float* o, float* states,
                                 int B, int T, int Hk, int Hv, int D, int nthreads);

namespace {

int g_fail = 0;

float rel_err(const std::vector<float>& a, const std::vector<float>& b) {
  float num = 0.f, den = 0.f;
  for (size_t i = 0; i < a.size(); ++i) {
    num = std::max(num, std::fabs(a[i] - b[i]));
    den = std::max(den, std::fabs(b[i]));
  }
  return num / (den > 0 ? den : 1.f);
}

void check(bool ok, const char* what) {
  std::printf("  [%s] %s\n", ok ? "ok" : "FAIL", what);
  if (!ok) ++g_fail;
}

void l2norm_rows(std::vector<float>& x, int D, float scale) {
  for (size_t r = 0; r < x.size() / D; ++r) {
    double ss = 0;
    for (int d = 0; d < D; ++d) ss += double(x[r * D + d]) * x[r * D + d];
    const float inv = 1.f / std::sqrt(float(ss) + 1e-6f);
    for (int d = 0; d < D; ++d) x[r * D + d] *= inv * scale;
  }
}

}  // namespace

int main() {
  if (!gdn::delta::available()) {
    std::printf("  [skip] no CUDA device\n");
    return 0;
  }
  std::mt19937 rng(0);
  std::normal_distribution<float> N01(0.f, 1.f);
  std::uniform_real_distribution<float> Ual(0.85f, 1.f), Ubt(0.f, 1.f);
  struct Case { int B, L, H; };
  const int D = 128;
  for (const Case c : {Case{1, 1, 48}, Case{1, 4, 48}, Case{1, 9, 48}, Case{2, 3, 16}, Case{1, 64, 48},
                       Case{1, 384, 8}}) {
    const size_t nqk = size_t(c.B) * c.L * c.H * D, ng = size_t(c.B) * c.L * c.H, ns = size_t(c.B) * c.H * D * D;
    std::vector<float> q(nqk), k(nqk), v(nqk), al(ng), bt(ng), S0(ns);
    for (auto& x : q) x = N01(rng);
    for (auto& x : k) x = N01(rng);
    for (auto& x : v) x = N01(rng);
    for (auto& x : al) x = Ual(rng);
    for (auto& x : bt) x = Ubt(rng);
    for (auto& x : S0) x = 0.1f * N01(rng);
    l2norm_rows(q, D, 1.f / std::sqrt(float(D)));
    l2norm_rows(k, D, 1.f);

    using gdn::DeviceArray;
    using gdn::DType;
    DeviceArray dq({c.B, c.L, c.H, D}, DType::F32), dk({c.B, c.L, c.H, D}, DType::F32),
        dv({c.B, c.L, c.H, D}, DType::F32), da({c.B, c.L, c.H}, DType::F32), db({c.B, c.L, c.H}, DType::F32),
        dS({c.B, c.H, D, D}, DType::F32);
    dq.upload(q.data()); dk.upload(k.data()); dv.upload(v.data());
    da.upload(al.data()); db.upload(bt.data()); dS.upload(S0.data());
    gdn::delta::Result got = gdn::delta::run(dq, dk, dv, da, db, &dS, /*collect=*/true);

    std::vector<float> o(nqk), S(ns), st(ns * c.L), ro(nqk), rS(ns), rst(ns * c.L);
    got.o.download(o.data());
    got.s_out.download(S.data());
    got.states.download(st.data());
    oracle_recurrent(q.data(), k.data(), v.data(), al.data(), bt.data(), S0.data(), rS.data(), ro.data(), rst.data(),
                     c.B, c.L, c.H, c.H, D, 0);
    const float eo = rel_err(o, ro), es = rel_err(S, rS), ec = rel_err(st, rst);
    char buf[160];
    std::snprintf(buf, sizeof(buf), "B=%d L=%3d H=%2d  out %.2e  state %.2e  collect (%d states) %.2e", c.B, c.L,
                  c.H, eo, es, c.L, ec);
    check(eo < 1e-5f && es < 1e-5f && ec < 1e-5f, buf);
  }
  // a state pool: one step of 3 sequences in slots {5, 0, 3} of 7 equals the dense step on those
  // states, bit for bit, and leaves the other slots untouched
  {
    using gdn::DeviceArray;
    using gdn::DType;
    const int B = 3, L = 1, Hk = 16, Hv = 48, n_slots = 7;
    const int slot_of[B] = {5, 0, 3};
    const size_t per = size_t(Hv) * D * D;
    std::vector<float> q(size_t(B) * L * Hk * D), k(q.size()), v(size_t(B) * L * Hv * D), a(size_t(B) * L * Hv),
        b(a.size()), A_log(Hv), dt(Hv), pool(per * n_slots), dense(per * B);
    for (auto& x : q) x = N01(rng);
    for (auto& x : k) x = N01(rng);
    for (auto& x : v) x = N01(rng);
    for (auto& x : a) x = N01(rng);
    for (auto& x : b) x = N01(rng);
    for (auto& x : A_log) x = 2.7f * Ubt(rng);
    for (auto& x : dt) x = Ubt(rng);
    for (auto& x : pool) x = 0.05f * N01(rng);
    for (int i = 0; i < B; ++i)
      std::copy(pool.begin() + per * slot_of[i], pool.begin() + per * (slot_of[i] + 1), dense.begin() + per * i);
    DeviceArray dq({B, L, Hk, D}, DType::F32), dk({B, L, Hk, D}, DType::F32), dv({B, L, Hv, D}, DType::F32),
        da({B, L, Hv}, DType::F32), db({B, L, Hv}, DType::F32), dA({Hv}, DType::F32), ddt({Hv}, DType::F32),
        dS({B, Hv, D, D}, DType::F32), dslots({B}, DType::I32);
    dq.upload(q.data()); dk.upload(k.data()); dv.upload(v.data()); da.upload(a.data()); db.upload(b.data());
    dA.upload(A_log.data()); ddt.upload(dt.data()); dS.upload(dense.data()); dslots.upload(slot_of);
    gdn::delta::StatePool sp(n_slots, Hv);
    sp.states().upload(pool.data());
    gdn::delta::Result want = gdn::delta::run_gated(dq, dk, dv, da, db, dA, ddt, &dS, false, true);
    gdn::delta::Result got = sp.step(dq, dk, dv, da, db, dA, ddt, dslots, false, true);
    std::vector<float> o1(size_t(B) * L * Hv * D), o2(o1.size()), S1(per * B), P2(pool.size());
    want.o.download(o1.data());
    want.s_out.download(S1.data());
    got.o.download(o2.data());
    sp.states().download(P2.data());
    bool same = o1 == o2;
    for (int i = 0; i < B; ++i)
      same = same && std::equal(S1.begin() + per * i, S1.begin() + per * (i + 1), P2.begin() + per * slot_of[i]);
    for (int s2 : {1, 2, 4, 6})
      same = same && std::equal(pool.begin() + per * s2, pool.begin() + per * (s2 + 1), P2.begin() + per * s2);
    check(same, "state pool step == dense step on the slots (bit for bit), other slots untouched");
  }
  // a rejected call throws with the library's message, like the reference's MLX errors
  bool threw = false;
  try {
    gdn::DeviceArray bad({1, 1, 1, 64}, gdn::DType::F32);
    gdn::delta::run(bad, bad, bad, bad, bad, nullptr);
  } catch (const std::runtime_error&) {
    threw = true;
  }
  check(threw, "Dk=64 is rejected with an exception");
  std::printf(g_fail ? "FAILURES ABOVE\n" : "ALL PASS\n");
  return g_fail ? 1 : 0;
}
