// Host-side construction of the IQ lattice search structures
// (quant_iq.rs:44-133 build_grid / expand_kgrid / grid_iq*).
//
// The reference builds, for every 2- or 3-bit lattice index u, either the
// grid index of the point (on-grid) or a list of the nearest grid points,
// sorted by (squared distance, index) and cut after `nwant` distinct
// distances.  The encoders only ever look up indices whose coordinates are
// reachable by their rounding (l in 0..2 for IQ2, 0..7 for IQ3), so the
// device copy is compacted to those: 3^8 = 6561 entries for IQ2 (base-3
// index) and all 4096 for IQ3.  The lists themselves are exactly the
// reference's for those points.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <vector>

#include "iq_tables.h"
#include "iq_host.h"

namespace shc {

namespace {
const uint16_t kgrid_2bit_256[256] = SH_KGRID_2BIT_256_DATA;
const uint16_t kgrid_2bit_512[512] = SH_KGRID_2BIT_512_DATA;
const uint16_t kgrid_2bit_1024[1024] = SH_KGRID_2BIT_1024_DATA;
const uint16_t kgrid_256[256] = SH_KGRID_256_DATA;
const uint16_t kgrid_512[512] = SH_KGRID_512_DATA;

struct Variant {
    const uint16_t *kgrid;
    int n, dim, bits, nwant;
};
const Variant kVariants[5] = {
    {kgrid_2bit_256, 256, 8, 2, 2},   // IQ2_XXS  quant_iq.rs:116
    {kgrid_2bit_512, 512, 8, 2, 2},   // IQ2_XS   quant_iq.rs:120
    {kgrid_2bit_1024, 1024, 8, 2, 1}, // IQ2_S    quant_iq.rs:124
    {kgrid_256, 256, 4, 3, 2},        // IQ3_XXS  quant_iq.rs:128
    {kgrid_512, 512, 4, 3, 3},        // IQ3_S    quant_iq.rs:132
};
}  // namespace

void build_iq_tables(int which, IqHostTable &t) {
    const Variant &v = kVariants[which];
    const int mask = (1 << v.bits) - 1;
    const int levels = v.bits == 2 ? 3 : 8;  // reachable l per coordinate
    int ncompact = 1;
    for (int k = 0; k < v.dim; k++) ncompact *= levels;
    t.grid_size = v.n;
    t.dim = v.dim;
    t.grid_coords.assign(v.kgrid, v.kgrid + v.n);
    // full-index -> grid index, as build_grid's first loop
    const int full = 1 << (v.bits * v.dim);
    std::vector<int32_t> onmap((size_t)full, -1);
    std::vector<int8_t> pts((size_t)v.n * 8);
    for (int i = 0; i < v.n; i++) {
        int index = 0;
        for (int k = 0; k < v.dim; k++) {
            const int l = (v.kgrid[i] >> (v.bits * k)) & mask;
            pts[(size_t)i * 8 + k] = (int8_t)(2 * l + 1);
            index |= l << (v.bits * k);
        }
        onmap[(size_t)index] = i;
    }
    t.kmap.assign((size_t)ncompact, 0);
    t.neighbours.clear();
    std::vector<std::pair<int32_t, uint16_t>> dist2((size_t)v.n);
    for (int c = 0; c < ncompact; c++) {
        int pos[8], u = 0, rem = c;
        for (int k = 0; k < v.dim; k++) {
            const int l = rem % levels;
            rem /= levels;
            pos[k] = 2 * l + 1;
            u |= l << (v.bits * k);
        }
        if (onmap[(size_t)u] >= 0) {
            t.kmap[(size_t)c] = onmap[(size_t)u];
            continue;
        }
        for (int j = 0; j < v.n; j++) {
            int d2 = 0;
            for (int k = 0; k < v.dim; k++) {
                const int d = pts[(size_t)j * 8 + k] - pos[k];
                d2 += d * d;
            }
            dist2[(size_t)j] = {d2, (uint16_t)j};
        }
        std::sort(dist2.begin(), dist2.end());
        t.kmap[(size_t)c] = -(int32_t)(t.neighbours.size() + 1);
        const size_t start = t.neighbours.size();
        t.neighbours.push_back(0);
        uint32_t cnt = 0;
        int nhave = 1;
        int32_t dcur = dist2[0].first;
        for (const auto &p : dist2) {
            if (p.first > dcur) {
                if (nhave == v.nwant) break;
                dcur = p.first;
                nhave++;
            }
            t.neighbours.push_back((uint32_t)p.second | ((uint32_t)v.kgrid[p.second] << 16));
            cnt++;
        }
        t.neighbours[start] = cnt;
    }
}

}  // namespace shc
