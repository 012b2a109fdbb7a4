// Host-built IQ lattice structures (see iq_host.cpp).
#pragma once
#include <cstdint>
#include <vector>

namespace shc {

struct IqHostTable {
    int grid_size = 0;
    int dim = 0;
    std::vector<uint32_t> grid_coords;  // packed lattice coordinates per grid point
    std::vector<int32_t> kmap;          // compact index -> grid index, or -(offset+1)
    std::vector<uint32_t> neighbours;   // [count, (grid index | coords << 16) ...] ...
};

// which: 0 IQ2_XXS, 1 IQ2_XS, 2 IQ2_S, 3 IQ3_XXS, 4 IQ3_S
void build_iq_tables(int which, IqHostTable &t);

}  // namespace shc
