// Header-only load of a GGUF flow pack through the reference API
// (SLatFlowModel::load with load_tensors = false): no device work.  Prints
// "ok <tensor_count> <model_channels> <num_blocks> <num_heads>" or
// "error <message>".
#include <iostream>
#include <string>

#include "pixal3d/slat_flow.h"

int main(int argc, char **argv) {
    if (argc != 3) {
        std::cerr << "usage: gguf_info <pack.gguf> <component>\n";
        return 2;
    }
    pixal3d::SLatFlowModel m;
    std::string e;
    if (!m.load(argv[1], argv[2], false, &e)) {
        std::cout << "error " << e << "\n";
        return 0;
    }
    const pixal3d::SLatFlowHParams &h = m.hparams();
    std::cout << "ok " << m.tensor_count() << " " << h.model_channels << " " << h.num_blocks << " " << h.num_heads
              << " " << (m.has_data() ? 1 : 0) << "\n";
    return 0;
}
