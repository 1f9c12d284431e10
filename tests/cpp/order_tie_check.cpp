// generate_balanced_window_order from fused3s.hpp compiled with
// F3S_REFERENCE_TIE_ORDER: the reference's exact permutation (std::sort with
// the reference's comparator, include/utils.cuh:48-59), on the host.
// Reads int32 window offsets (nrw + 1) from argv[1], writes the int32 order
// to argv[2].  Needs no GPU.
#define F3S_REFERENCE_TIE_ORDER
#include "fused3s.hpp"

#include <cstdio>
#include <vector>

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 3;
    std::vector<int> off;
    int v;
    while (std::fread(&v, sizeof v, 1, f) == 1) off.push_back(v);
    std::fclose(f);
    if (off.empty()) return 4;
    blockSparseFormat fmt;
    fmt.num_row_windows = (int)off.size() - 1;
    fmt.window_offsets = off;
    std::vector<int> order = generate_balanced_window_order(fmt);
    FILE* o = std::fopen(argv[2], "wb");
    if (!o) return 5;
    std::fwrite(order.data(), sizeof(int), order.size(), o);
    std::fclose(o);
    return 0;
}
