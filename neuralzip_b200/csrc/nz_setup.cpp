// Setup-time chunk clustering on the host.
//
// Restates the clustering rule of the reference's setup
// (neuralzip/setup.py:91-141): chunks are visited in checkpoint order; a
// chunk joins the nearest existing cluster of its class (same dtype and same
// forced label), by the base-2 Jensen-Shannon distance between its exponent
// distribution and the cluster centroid (ties: the earliest cluster), if that
// distance is at most the threshold or the chunk's label forces it; else it
// opens a cluster. The centroid is the weight-averaged distribution of the
// cluster's chunks, updated after every assignment. The reference scans the
// clusters in Python once per chunk; here the whole pass is one native loop
// over flat arrays. Distances use libm's log2 and a plain left-to-right sum,
// so a chunk whose distance lies within rounding of the threshold may fall
// on the other side of it than in the reference (which only changes which
// codebook codes that chunk, never what decodes).

#include "nz_b200.h"
#include "nz_internal.h"

#include <cmath>
#include <cstring>
#include <vector>

namespace {

double js_distance(const double* a, const double* b, uint32_t bins) {
    double left = 0.0, right = 0.0;
    for (uint32_t k = 0; k < bins; ++k) {
        const double m = 0.5 * (a[k] + b[k]);
        if (a[k] > 0.0) left += a[k] * std::log2(a[k] / m);
        if (b[k] > 0.0) right += b[k] * std::log2(b[k] / m);
    }
    const double divergence = 0.5 * left + 0.5 * right;
    return std::sqrt(divergence > 0.0 ? divergence : 0.0);
}

}  // namespace

extern "C" {

int nz_cluster_chunks(const double* distributions, const double* weights, const int32_t* classes,
                      const uint8_t* forced, uint64_t count, uint32_t bins, double threshold, int32_t share,
                      uint32_t* assign, double* centroids, uint64_t cap_clusters, uint64_t* n_clusters) {
    NZ_GUARD({
        if (count && (!distributions || !weights || !classes || !forced || !assign))
            throw nz::Error(NZ_EVALUE, "Null clustering argument.");
        if (!n_clusters || (cap_clusters && !centroids) || bins == 0)
            throw nz::Error(NZ_EVALUE, "Null clustering output.");
        std::vector<int32_t> cluster_class;
        std::vector<double> cluster_weight;
        for (uint64_t i = 0; i < count; ++i) {
            const double* d = distributions + i * bins;
            int64_t best = -1;
            double best_distance = 0.0;
            if (share) {
                for (uint64_t c = 0; c < cluster_class.size(); ++c) {
                    if (cluster_class[c] != classes[i]) continue;
                    const double distance = js_distance(d, centroids + c * bins, bins);
                    if (best < 0 || distance < best_distance) best = static_cast<int64_t>(c), best_distance = distance;
                }
            }
            if (best < 0 || (!forced[i] && best_distance > threshold)) {
                if (cluster_class.size() >= cap_clusters) throw nz::Error(NZ_EOVERFLOW, "Too many clusters.");
                best = static_cast<int64_t>(cluster_class.size());
                cluster_class.push_back(classes[i]);
                cluster_weight.push_back(0.0);
                std::memcpy(centroids + best * bins, d, bins * sizeof(double));
            }
            double* centroid = centroids + best * bins;
            const double w = weights[i], total = cluster_weight[best] + w;
            for (uint32_t k = 0; k < bins; ++k) centroid[k] = (centroid[k] * cluster_weight[best] + d[k] * w) / total;
            cluster_weight[best] = total;
            assign[i] = static_cast<uint32_t>(best);
        }
        *n_clusters = cluster_class.size();
    })
}

}  // extern "C"
