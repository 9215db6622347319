// property.cuh -- the verdict of one box from its specification bounds,
// shared by the host entry point and the batched device kernel.
#pragma once

#include <cstdint>

#include "luna_b200.h"

namespace lb200 {

// Status of one box whose rows of C.y are bounded by [lb, ub]
// (LunaMain.cpp:60-135 evaluatePropertyStatus, with
// OutputConstraintSet::evaluateORBranches, OutputConstraint.cpp:187-278).
// The property says "the counterexample region C.y <= thresholds is
// reachable":
//   n_branches == 0 (a conjunction): UNSAT when some row has lb - thr > 0;
//     SAT when every row has ub - thr <= 0;
//   n_branches  > 0 (a disjunction of conjunctions, row r in branch
//     branch[r]): UNSAT when every branch has a row with lb - thr > 0; SAT
//     when some non-empty branch has no row with ub - thr > 0.
// Differences are taken in fp32 before the comparison, as Luna does; the
// two forms treat NaN differently (a NaN upper bound never refutes a
// conjunction but does not stop a branch from refuting), as Luna does.
__host__ __device__ inline int box_status(const float* lb, const float* ub, const float* thr,
                                          const int32_t* branch, int64_t nspec, int32_t n_branches) {
    if (nspec <= 0) return LB200_STATUS_UNKNOWN;
    if (n_branches <= 0) {
        bool broken = false, all_sat = true;
        for (int64_t r = 0; r < nspec; ++r) {
            const float dl = lb[r] - thr[r];
            const float du = ub[r] - thr[r];
            broken |= dl > 0.0f;
            all_sat &= du <= 0.0f;
        }
        if (broken) return LB200_STATUS_UNSAT;
        return all_sat ? LB200_STATUS_SAT : LB200_STATUS_UNKNOWN;
    }
    bool all_disproved = true, any_always_sat = false;
    for (int32_t b = 0; b < n_branches; ++b) {
        bool rows = false, disproved = false, always_sat = true;
        for (int64_t r = 0; r < nspec; ++r) {
            if (branch[r] != b) continue;
            rows = true;
            disproved |= lb[r] - thr[r] > 0.0f;
            if (ub[r] - thr[r] > 0.0f) always_sat = false;
        }
        if (!rows) always_sat = false;
        all_disproved &= disproved;
        any_always_sat |= always_sat;
    }
    if (all_disproved) return LB200_STATUS_UNSAT;
    return any_always_sat ? LB200_STATUS_SAT : LB200_STATUS_UNKNOWN;
}

// TorchModel::isSpecVerified (TorchModel.cpp:616-651) from the lower bounds
// alone: the conjunction is broken by one row, every branch of a
// disjunction by one of its rows.
__host__ __device__ inline bool box_verified(const float* lb, const float* thr, const int32_t* branch, int64_t nspec,
                                             int32_t n_branches) {
    if (nspec <= 0) return false;
    if (n_branches <= 0) {
        for (int64_t r = 0; r < nspec; ++r)
            if (lb[r] - thr[r] > 0.0f) return true;
        return false;
    }
    for (int32_t b = 0; b < n_branches; ++b) {
        bool disproved = false;
        for (int64_t r = 0; r < nspec && !disproved; ++r)
            disproved = branch[r] == b && lb[r] - thr[r] > 0.0f;
        if (!disproved) return false;
    }
    return true;
}

}  // namespace lb200
