// plan.hpp -- host-side model description and planning helpers.
#pragma once

#include "internal.hpp"
#include "neighbors.hpp"

#include <string>
#include <vector>

namespace mtpb {

// Owned host copy of a linear MTP model (mtpb_model_view).
struct ModelHost {
    int K = 0, mu = 0, R = 0, split = 0, M = 0;
    double scaling = 1.0;
    std::vector<double> min_dist, max_dist;
    std::vector<int> basic;    // [nb*4]
    std::vector<int> times;    // [T*4]
    std::vector<int> mapping;  // [S]
    std::vector<double> radial, species, moment;
    std::vector<RadialFamily> family;   // empty: RBChebyshev; else 1 or K*K (split)
    int nb() const { return (int)basic.size() / 4; }
    int T() const { return (int)times.size() / 4; }
    int S() const { return (int)mapping.size(); }
    int pairs() const { return K * K; }
    double pair_min(int p) const { return split ? min_dist[p] : min_dist[0]; }
    double pair_max(int p) const { return split ? max_dist[p] : max_dist[0]; }
    RadialFamily pair_family(int p) const
    {
        return family.empty() ? RadialFamily{} : family[split && family.size() > 1 ? p : 0];
    }
    double cutoff() const
    {
        double c = 0;
        for (double v : max_dist)
            c = v > c ? v : c;
        return c;
    }
    int radial_count() const { return K * K * mu * R; }
    int coeff_count() const { return radial_count() + K + S(); }
};

bool validate_model(const ModelHost &m, std::string *err);
int select_shape(const ModelHost &m, std::string *err);
bool build_slot_map(const ModelHost &m, int shape, std::vector<int> &slot_of_basic,
                    std::string *err);
bool build_dag_plan(const ModelHost &m, int shape, const std::vector<int> &slot_of_basic,
                    DagPlan &plan, std::string *err);

} // namespace mtpb
