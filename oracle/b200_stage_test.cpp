// Test infrastructure: the boundary seen from the reference's side.  Opens a GGUF file with
// the reference's own loader, runs the same prompt through the reference's Model (stage v2,
// src/model.hpp:24-50) and through ModelB200 (b200_stage.hpp: the binding a maintainer adds,
// built on libtinferno_b200.so), greedy-decodes n steps with each, and compares.
//
//   b200_stage_test MODEL.gguf MAX_SEQ N_DECODE TOKEN...
//
// Prints one JSON line {"tokens_equal":..., "max_abs_logit_diff":..., ...} and exits 0 when the
// greedy ids are identical and every step's logits agree within 1e-2 (the engine's parity
// tolerance), 1 when they do not, 2 on an error.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <thread>
#include <vector>

#include "b200_stage.hpp"
#include "model.hpp"
#include "sampler.hpp"

using namespace tinf;

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s MODEL.gguf MAX_SEQ N_DECODE TOKEN...\n", argv[0]);
        return 2;
    }
    try {
        const std::string path = argv[1];
        const int max_seq = std::atoi(argv[2]);
        const int n_decode = std::atoi(argv[3]);
        std::vector<int> prompt;
        for (int i = 4; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));

        int hw = (int)std::thread::hardware_concurrency();
        RunConfig rc = stage_preset("v2", hw > 0 ? hw : 4);
        rc.max_seq = max_seq;
        Model ref(path, rc);  // the reference engine
        GGUF g(path);         // the reference's loader feeds the B200 stage
        ModelB200 b200(g, rc);
        if (b200.n_vocab() != ref.n_vocab()) throw std::runtime_error("n_vocab differs");

        const int V = ref.n_vocab();
        std::vector<float> lr(V), lb(V);
        ref.prefill(prompt.data(), (int)prompt.size(), lr.data());
        b200.prefill(prompt.data(), (int)prompt.size(), lb.data());
        std::vector<int> ids_r, ids_b;
        double max_diff = 0.0;
        for (int s = 0; s <= n_decode; ++s) {
            for (int i = 0; i < V; ++i) max_diff = std::max(max_diff, (double)std::fabs(lr[i] - lb[i]));
            const int tr = sample_greedy(lr.data(), V);
            const int tb = sample_greedy(lb.data(), V);
            ids_r.push_back(tr);
            ids_b.push_back(tb);
            if (s == n_decode) break;
            ref.decode(tr, lr.data());
            b200.decode(tb, lb.data());
        }
        const bool pos_equal = ref.n_pos() == b200.n_pos();
        // the device greedy loop from the same prefill, against the reference's ids
        b200.reset();
        b200.prefill(prompt.data(), (int)prompt.size(), lb.data());
        std::vector<int> gen = b200.generate_greedy(sample_greedy(lb.data(), V), n_decode + 1);
        const bool gen_equal = gen.size() <= ids_r.size() && std::equal(gen.begin(), gen.end(), ids_r.begin());
        const bool equal = ids_r == ids_b;
        std::printf("{\"tokens_equal\": %s, \"generate_equal\": %s, \"n_pos_equal\": %s, \"steps\": %d, "
                    "\"max_abs_logit_diff\": %.3e, \"first_ids\": [%d, %d, %d]}\n",
                    equal ? "true" : "false", gen_equal ? "true" : "false", pos_equal ? "true" : "false",
                    (int)ids_r.size(), max_diff, ids_r[0], ids_r.size() > 1 ? ids_r[1] : -1,
                    ids_r.size() > 2 ? ids_r[2] : -1);
        return (equal && gen_equal && pos_equal && max_diff < 1e-2) ? 0 : 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 2;
    }
}
