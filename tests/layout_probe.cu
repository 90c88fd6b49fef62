// Host-only probe of the slab layouts the launches use (test infrastructure
// for tests/test_layout.py): prints one JSON object for the extents and the
// layout choice given on the command line,
//   layout_probe H W neutral capacity types offsets aligned bots hbm compact
// where `hbm` selects the rules-only rows kept in HBM (kRulesRows).
#include "../nanorts_b200/csrc/step.cu"

#include <cstdio>
#include <cstdlib>

int main(int argc, char** argv) {
    if (argc != 11) {
        std::fprintf(stderr, "usage: layout_probe H W neutral capacity types offsets aligned bots hbm compact\n");
        return 2;
    }
    NrtsExtents x{};
    x.height = std::atoi(argv[1]);
    x.width = std::atoi(argv[2]);
    x.neutral = std::atoi(argv[3]);
    x.capacity = std::atoi(argv[4]);
    x.types = std::atoi(argv[5]);
    x.offsets = std::atoi(argv[6]);
    const bool aligned = std::atoi(argv[7]) != 0, bots = std::atoi(argv[8]) != 0;
    const bool hbm = std::atoi(argv[9]) != 0, compact = std::atoi(argv[10]) != 0;
    const Layout L = make_layout(&x, aligned, bots, hbm ? nrts::kRulesRows : 0u, compact);
    std::printf("{\"leaf_off\": [");
    for (int k = 0; k < nrts::kSlabLeaves; ++k) std::printf("%s%d", k ? ", " : "", L.leaf_off[k]);
    std::printf("], \"row_bytes\": [");
    for (int k = 0; k < nrts::kSlabLeaves; ++k) std::printf("%s%d", k ? ", " : "", L.row_bytes[k]);
    std::printf("], \"scal_off\": %d, \"list_off\": %d, \"order_off\": %d, \"serial_off\": %d, \"scan_off\": %d, \"conf_off\": %d, "
                "\"key_off\": %d, \"info_off\": %d, \"rank_off\": %d, \"count_off\": %d, \"free_off\": %d, \"member_key_off\": %d, "
                "\"ret_off\": %d, \"word_off\": %d, \"rows_off\": %d, \"mask_off\": %d, \"carry_off\": %d, \"cmd_off\": %d, "
                "\"bot_off\": %d, \"bot_bytes\": %d, \"bar_off\": %d, \"slab_bytes\": %d, \"header_bytes\": %d, \"claim_words\": %d}\n",
                L.scal_off, L.list_off, L.order_off, L.serial_off, L.scan_off, L.conf_off, L.key_off, L.info_off, L.rank_off,
                L.count_off, L.free_off, L.member_key_off, L.ret_off, L.word_off, L.rows_off, L.mask_off, L.carry_off, L.cmd_off,
                L.bot_off, bots ? nrts::bot_layout(x.capacity, x.neutral + 2 * x.capacity, x.height * x.width, 0).bytes : 0,
                L.bar_off, L.slab_bytes, L.header_bytes, nrts::claim_words(x.height * x.width, compact));
    return 0;
}
