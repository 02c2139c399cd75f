// stork.cpp -- the STORK4 solver (src/solvers/solver-stork.h) on device buffers: the step history,
// the derivative order with its stability guards, the ROCK4 degree choice, the host-side scalar
// recurrence, the adaptive halving of the sub step count on a non-finite result and the Euler
// fallback, in the reference's order. The ROCK4 tables (degrees, finishing coefficients,
// recurrence coefficients) are the caller's: the reference compiles them in
// (solver-stork4-constants.h), and this library takes them through acb_stork4_tables.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/acb_models.h"
#include "host_common.h"
#include "stork.h"
#include "weights.h"

using namespace acb;

struct acb_stork4 {
    int                 device   = 0;
    int64_t             n        = 0;
    int                 substeps = 10;  // SolverState::stork_substeps
    std::vector<int>    ms;
    std::vector<double> fpa, fpb, recf;  // [len][6], [len][4], recurrence
    int                 step_index = 0;
    int                 nh         = 0;  // history records held (at most 2 are read)
    float               dt_last = 0.0f, dt_prev = 0.0f;
    DevBuf              h_last, h_prev, dv, d2v, xn, coef, part, sums, flag;
    int                 nblk = 0;
    std::vector<float>  coef_h;

    acb_status push_history(const float * vt, float dt, cudaStream_t s) {
        // the newest record becomes hist.back(), the one before hist[size-2]
        std::swap(h_last.p, h_prev.p);
        std::swap(h_last.bytes, h_prev.bytes);
        dt_prev = dt_last;
        dt_last = dt;
        nh      = nh < 3 ? nh + 1 : 3;
        return cudaMemcpyAsync(h_last.p, vt, (size_t) n * 4, cudaMemcpyDeviceToDevice, s) == cudaSuccess ?
                   ACB_OK :
                   ACB_ERR_CUDA;
    }

    // _rock4_mdegr (solver-stork.h:138-158)
    void mdegr(int s, int & mdeg, int & mz, int & mr) const {
        int mp1 = 1;
        mdeg    = s;
        mz      = 0;
        mr      = 0;
        for (size_t i = 0; i < ms.size(); i++) {
            if (ms[i] >= s) {
                mdeg = ms[i];
                mz   = (int) i;
                mr   = mp1 - 1;
                return;
            }
            mp1 += ms[i] * 2 - 1;
        }
        mz   = (int) ms.size() - 1;
        mdeg = ms[(size_t) mz];
        mr   = mp1 - 1;
    }

    acb_status euler(float * xt, const float * vt, float dt, cudaStream_t s);
    acb_status step(float * xt, const float * vt, float t_curr, float t_prev, cudaStream_t s);
};

acb_status acb_stork4::euler(float * xt, const float * vt, float dt, cudaStream_t s) {
    // xt -= vt * dt: acb_dit_euler's arithmetic with tt = {dt, dt, 0}, which gives xt - vt * dt
    const float tt[3] = { dt, dt, 0.0f };
    if (cudaMemcpyAsync(coef.p, tt, sizeof(tt), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return acb_dit_euler(xt, vt, coef.as<float>(), 0, nullptr, n, (acb_stream_t) s);
}

acb_status acb_stork4::step(float * xt, const float * vt, float t_curr, float t_prev, cudaStream_t s) {
    const float dt = t_curr - t_prev;
    if (step_index == 0) {  // bootstrap: plain Euler, no history yet
        ACB_TRY(euler(xt, vt, dt, s));
        ACB_TRY(push_history(vt, dt, s));
        step_index = 1;
        return cudaStreamSynchronize(s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
    }
    // _stork_compute_derivatives (solver-stork.h:72-127)
    int         order = 0;
    const float h1    = dt_last;
    if (nh >= 1 && h1 != 0.0f) {
        const float  h2    = dt_prev;
        const double h1d = (double) h1, h2d = (double) h2;
        const bool   want2 = nh >= 2 && h2 != 0.0f && !(fabs(h1d * h2d * (h1d + h2d)) < 1e-30);
        ACB_TRY(stork4_derivs(vt, h_last.as<float>(), h1, want2 ? h_prev.as<float>() : nullptr, h2, want2 ? 1 : 0, n,
                              dv.as<float>(), d2v.as<float>(), part.as<double>(), nblk, sums.as<double>(), s));
        double sm[3] = { 0, 0, 0 };
        if (cudaMemcpyAsync(sm, sums.p, sizeof(sm), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        const double vt_rms = sqrt(sm[0] / (double) n), dv_rms = sqrt(sm[1] / (double) n);
        if (vt_rms > 0.0 && dv_rms * fabs(h1) > 5.0 * vt_rms) {
            order = 0;
        } else if (nh < 2 || h2 == 0.0f || !want2) {
            order = 1;
        } else {
            const double d2v_rms = sqrt(sm[2] / (double) n);
            order                = (vt_rms > 0.0 && d2v_rms * h1 * h1 > 5.0 * vt_rms) ? 1 : 2;
        }
    }
    // adaptive sub stepping: substeps, halved on a non-finite result down to 2
    bool ok = false;
    for (int sub = substeps >= 2 ? substeps : 2; sub >= 2 && !ok; sub /= 2) {
        int s_eff = sub > ms.back() ? ms.back() : sub;
        int mdeg, mz, mr;
        mdegr(s_eff, mdeg, mz, mr);
        // the scalar recurrence (solver-stork.h:189-215) and the finishing offsets (:224-262)
        coef_h.assign((size_t) (mdeg + 1) * 4, 0.0f);
        const float t1_first = -dt * (float) recf[(size_t) mr];
        float       ci1 = t_curr + t1_first, ci2 = ci1, ci3 = t_curr;
        for (int j = 2; j <= mdeg; j++) {
            const float diff  = ci1 - t_curr;
            const float temp1 = -dt * (float) recf[(size_t) (mr + 2 * (j - 2) + 1)];
            const float temp3 = -(float) recf[(size_t) (mr + 2 * (j - 2) + 2)];
            const float temp2 = 1.0f - temp3;
            const float c_new = temp1 + temp2 * ci2 + temp3 * ci3;
            float *     c     = &coef_h[(size_t) j * 4];
            c[0] = temp1, c[1] = temp2, c[2] = temp3, c[3] = diff;
            ci3 = ci2;
            ci2 = c_new;
            ci1 = c_new;
        }
        const double * A    = &fpa[(size_t) mz * 6];
        const double * B    = &fpb[(size_t) mz * 4];
        const float    fpa0 = -dt * (float) A[0], fpa1 = -dt * (float) A[1], fpa2 = -dt * (float) A[2];
        const float    fpa3 = -dt * (float) A[3], fpa4 = -dt * (float) A[4], fpa5 = -dt * (float) A[5];
        float          diff4[4], fpb4[4];
        diff4[0] = ci1 - t_curr;
        diff4[1] = (ci1 + fpa0) - t_curr;
        diff4[2] = ((ci1 + fpa1) + fpa2) - t_curr;
        diff4[3] = (((ci1 + fpa3) + fpa4) + fpa5) - t_curr;
        for (int k = 0; k < 4; k++) {
            fpb4[k] = -dt * (float) B[k];
        }
        const size_t cb = coef_h.size() * 4;
        if ((coef.bytes < cb && coef.alloc(cb, false) != ACB_OK) ||
            cudaMemcpyAsync(coef.p, coef_h.data(), cb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemsetAsync(flag.p, 0, 4, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        ACB_TRY(stork4_substep(xt, vt, dv.as<float>(), d2v.as<float>(), order, coef.as<float>(), mdeg, t1_first,
                               diff4, fpb4, n, xn.as<float>(), flag.as<int>(), s));
        int bad = 0;
        if (cudaMemcpyAsync(&bad, flag.p, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        ok = bad == 0;
    }
    if (ok) {
        if (cudaMemcpyAsync(xt, xn.p, (size_t) n * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    } else {
        ACB_TRY(euler(xt, vt, dt, s));  // last resort (solver-stork.h:300-306)
    }
    ACB_TRY(push_history(vt, dt, s));
    step_index++;
    return cudaStreamSynchronize(s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

extern "C" acb_status acb_stork4_create(const acb_stork4_tables * t, int64_t n, int substeps, acb_stork4 ** out) {
    if (!t || !out || n <= 0 || !t->ms || t->ms_len <= 0 || !t->fpa || !t->fpb || !t->recf || t->recf_len <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    std::unique_ptr<acb_stork4> st(new acb_stork4());
    cudaGetDevice(&st->device);
    st->n        = n;
    st->substeps = substeps > 0 ? substeps : 10;
    st->ms.assign(t->ms, t->ms + t->ms_len);
    st->fpa.assign(t->fpa, t->fpa + (size_t) t->ms_len * 6);
    st->fpb.assign(t->fpb, t->fpb + (size_t) t->ms_len * 4);
    st->recf.assign(t->recf, t->recf + t->recf_len);
    // every recurrence index the degree table can reach must exist
    int need = 0, mp1 = 1;
    for (int i = 0; i < t->ms_len; i++) {
        if (t->ms[i] <= 0 || (i > 0 && t->ms[i] <= t->ms[i - 1])) {
            set_last_error("STORK4 degree table must be positive and increasing");
            return ACB_ERR_INVALID_ARG;
        }
        need = mp1 - 1 + 2 * (t->ms[i] - 2) + 3;
        mp1 += t->ms[i] * 2 - 1;
    }
    if (need > t->recf_len) {
        set_last_error("STORK4 recurrence table shorter than the degree table needs");
        return ACB_ERR_INVALID_ARG;
    }
    st->nblk       = 296;
    const size_t b = (size_t) n * 4;
    if (st->h_last.alloc(b) != ACB_OK || st->h_prev.alloc(b) != ACB_OK || st->dv.alloc(b) != ACB_OK ||
        st->d2v.alloc(b) != ACB_OK || st->xn.alloc(b) != ACB_OK || st->coef.alloc(4096, false) != ACB_OK ||
        st->part.alloc((size_t) st->nblk * 3 * 8) != ACB_OK || st->sums.alloc(3 * 8) != ACB_OK ||
        st->flag.alloc(4) != ACB_OK) {
        set_last_error("STORK4 buffers allocation failed");
        return ACB_ERR_OOM;
    }
    *out = st.release();
    return ACB_OK;
}

extern "C" acb_status acb_stork4_step(acb_stork4 * st, float * xt, const float * vt, float t_curr, float t_prev,
                                      acb_stream_t stream) {
    if (!st || !xt || !vt) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(st->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return st->step(xt, vt, t_curr, t_prev, (cudaStream_t) stream);
}

extern "C" void acb_stork4_reset(acb_stork4 * st) {
    if (st) {
        st->step_index = 0;
        st->nh         = 0;
        st->dt_last = st->dt_prev = 0.0f;
    }
}

extern "C" int acb_stork4_step_index(const acb_stork4 * st) {
    return st ? st->step_index : -1;
}

extern "C" void acb_stork4_free(acb_stork4 * st) {
    if (st) {
        cudaSetDevice(st->device);
        delete st;
    }
}
