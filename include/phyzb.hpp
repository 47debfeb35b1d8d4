// phyzb.hpp — C++ host side of libphyzb200, mirroring phyz-gpu's BatchSim.
//
// phyz's batched path is driven from Rust through `BatchSim<B>`
// (crates/phyz-gpu/src/cuda/mod.rs:430-1377); this header gives C++ hosts the
// same surface over the C ABI in phyzb.h. Errors follow the reference's two
// styles: the try_* methods return a phyzb::Result (the reference's
// Result<_, String>), the plain methods throw phyzb::Error where the
// reference panics (`step`, `load_states`, `readback_states`).
//
// Header-only; link with libphyzb200.so.
#pragma once

#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "phyzb.h"

namespace phyzb {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Result<T, String>: ok() or the failing call's message.
template <class T>
struct Result {
    bool ok_ = false;
    T value{};
    int code = PHYZB_OK;
    std::string error;
    bool ok() const { return ok_; }
    const T& unwrap() const {
        if (!ok_) throw Error(code, error);
        return value;
    }
};
struct Unit {};

inline Result<Unit> status(int rc) {
    Result<Unit> r;
    r.ok_ = rc == PHYZB_OK;
    r.code = rc;
    if (!r.ok_) r.error = phyzb_last_error();
    return r;
}
inline void check(int rc) {
    if (rc != PHYZB_OK) throw Error(rc, phyzb_last_error());
}

struct PdDof {
    int q_index, v_index;
    double kp, kd, max_force;
};
struct BodyContactGains {
    double stiffness, damping;
};

class BatchSim {
   public:
    // BatchSim::new / on_device (cuda/mod.rs:470-485): Err without a driver.
    static Result<BatchSim> on_device(const phyzb_model& model, int64_t nworld, int ordinal,
                                      int precision = PHYZB_F64) {
        Result<BatchSim> r;
        phyzb_sim* h = nullptr;
        r.code = phyzb_create(&model, nworld, ordinal, precision, &h);
        if (r.code != PHYZB_OK) {
            r.error = phyzb_last_error();
            return r;
        }
        r.ok_ = true;
        r.value = BatchSim(h, nworld, model);
        return r;
    }
    static Result<BatchSim> create(const phyzb_model& model, int64_t nworld, int precision = PHYZB_F64) {
        return on_device(model, nworld, 0, precision);
    }

    BatchSim() = default;
    BatchSim(const BatchSim&) = delete;
    BatchSim& operator=(const BatchSim&) = delete;
    BatchSim(BatchSim&& o) noexcept { *this = std::move(o); }
    BatchSim& operator=(BatchSim&& o) noexcept {
        if (this != &o) {
            reset();
            h_ = o.h_;
            nworld_ = o.nworld_;
            nv_ = o.nv_;
            nb_ = o.nb_;
            npd_ = o.npd_;
            o.h_ = nullptr;
        }
        return *this;
    }
    ~BatchSim() { reset(); }

    int64_t nworld() const { return nworld_; }
    int nv() const { return nv_; }
    int nbodies() const { return nb_; }
    phyzb_sim* raw() const { return h_; }

    Result<Unit> set_model(const phyzb_model& m) { return status(phyzb_set_model(h_, &m)); }

    // contact (cuda/mod.rs:596-700)
    Result<int> enable_ground_contact(double ground, double k, double d, double mu) {
        int32_t n = 0;
        return count(phyzb_enable_ground_contact(h_, ground, k, d, mu, &n), n);
    }
    Result<int> enable_ground_contact_per_body(double ground, double mu, const std::vector<BodyContactGains>& g) {
        std::vector<double> k, d;
        for (const auto& x : g) {
            k.push_back(x.stiffness);
            d.push_back(x.damping);
        }
        int32_t n = 0;
        return count(phyzb_enable_ground_contact_per_body(h_, ground, mu, k.data(), d.data(), &n), n);
    }
    int collidable_bodies() const { return phyzb_collidable_bodies(h_); }

    // PD (cuda/mod.rs:771-801)
    Result<Unit> enable_pd_control(const std::vector<PdDof>& dofs) {
        std::vector<phyzb_pd_dof> c;
        for (const auto& d : dofs) c.push_back(phyzb_pd_dof{d.q_index, d.v_index, d.kp, d.kd, d.max_force});
        Result<Unit> r = status(phyzb_enable_pd(h_, c.data(), (int32_t)c.size()));
        if (r.ok()) npd_ = (int)c.size();
        return r;
    }
    Result<Unit> set_position_targets(const std::vector<std::vector<double>>& t) {
        return status(phyzb_set_position_targets(h_, rows(t, npd_).data()));
    }

    // state (cuda/mod.rs:804-821): rows zero-padded / truncated like pack_rows
    void load_states(const std::vector<std::vector<double>>& q, const std::vector<std::vector<double>>& v,
                     const std::vector<std::vector<double>>* ctrl = nullptr) {
        std::vector<double> c = ctrl ? rows(*ctrl, nv_) : std::vector<double>();
        check(phyzb_load_states(h_, rows(q, nv_).data(), rows(v, nv_).data(), ctrl ? c.data() : nullptr));
    }
    void set_controls(const std::vector<std::vector<double>>& ctrl) {
        check(phyzb_set_controls(h_, rows(ctrl, nv_).data()));
    }

    // stepping (cuda/mod.rs:818-875)
    void step() { check(phyzb_step(h_, 1)); }
    Result<Unit> try_step() { return status(phyzb_step(h_, 1)); }
    Result<Unit> step_many(int n) { return status(phyzb_step(h_, n)); }
    // PHYZB_SPECIALIZE_OFF / _ON / _AUTO: the rollout kernel compiled at run
    // time for this model (phyzb_set_kernel_specialization)
    void set_kernel_specialization(int mode) { check(phyzb_set_kernel_specialization(h_, mode)); }

    // readback (cuda/mod.rs:978-996): rows of nv
    std::pair<std::vector<std::vector<double>>, std::vector<std::vector<double>>> readback_states() {
        std::vector<double> q((size_t)nworld_ * nv_), v((size_t)nworld_ * nv_);
        check(phyzb_readback_states(h_, q.data(), v.data()));
        return {split(q, nv_), split(v, nv_)};
    }
    Result<std::vector<double>> readback_contacts() {
        Result<std::vector<double>> r;
        r.value.resize((size_t)nworld_ * nb_ * PHYZB_CONTACT_STRIDE);
        r.code = phyzb_readback_contacts(h_, r.value.data());
        r.ok_ = r.code == PHYZB_OK;
        if (!r.ok_) r.error = phyzb_last_error();
        return r;
    }

   private:
    BatchSim(phyzb_sim* h, int64_t nworld, const phyzb_model& m) : h_(h), nworld_(nworld), nb_(m.nbodies) {
        phyzb_device_view dv;
        if (phyzb_device_view_get(h, &dv) == PHYZB_OK) nv_ = dv.nv;
    }
    void reset() {
        if (h_) phyzb_destroy(h_);
        h_ = nullptr;
    }
    Result<int> count(int rc, int n) {
        Result<int> r;
        r.code = rc;
        r.ok_ = rc == PHYZB_OK;
        if (r.ok_)
            r.value = n;
        else
            r.error = phyzb_last_error();
        return r;
    }
    std::vector<double> rows(const std::vector<std::vector<double>>& a, int width) const {
        std::vector<double> out((size_t)nworld_ * width, 0.0);
        for (size_t w = 0; w < a.size() && (int64_t)w < nworld_; w++)
            for (size_t k = 0; k < a[w].size() && (int)k < width; k++) out[w * width + k] = a[w][k];
        return out;
    }
    std::vector<std::vector<double>> split(const std::vector<double>& flat, int width) const {
        std::vector<std::vector<double>> out((size_t)nworld_);
        for (int64_t w = 0; w < nworld_; w++) out[w].assign(flat.begin() + w * width, flat.begin() + (w + 1) * width);
        return out;
    }

    phyzb_sim* h_ = nullptr;
    int64_t nworld_ = 0;
    int nv_ = 0, nb_ = 0, npd_ = 0;
};

}  // namespace phyzb
