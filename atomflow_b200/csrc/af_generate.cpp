// af_generate -- greedy decoding from the command line on the C ABI of
// libatomflow_b200.so: the reference's autoregressive loop (src/main.cu:
// 228-276) and its graph TPOT measurement (src/main.cu:92-150), in C++ with
// no Python.
//
//   af_generate --model M.bin --prompt ids.txt [--steps 64] [--mode exact|fast]
//               [--max-seq 4096] [--true-argmax] [--tpot-steps 0]
//
// The prompt file holds token ids (whitespace separated).  Each prompt token is
// fed at positions 0, 1, ... (teacher forcing); then `steps` greedy tokens
// follow from the last prompt position + 1.  Output: one line per greedy
// token, then "tpot_ms <v>" when --tpot-steps > 0 (replays of the captured
// step at the final position, CUDA events on the engine's stream).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "../../include/atomflow_b200.h"

static int fail(const char* what, af_status st) {
    std::fprintf(stderr, "af_generate: %s: %s %s\n", what, af_status_string(st),
                 st == AF_ERR_CUDA ? af_last_cuda_error() : "");
    return 1;
}

int main(int argc, char** argv) {
    std::string model, prompt;
    int steps = 64, max_seq = 4096, tpot_steps = 0;
    af_engine_mode mode = AF_ENGINE_EXACT;
    af_argmax_mode amode = AF_ARGMAX_REF_COMPAT;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&]() -> const char* { return i + 1 < argc ? argv[++i] : ""; };
        if (a == "--model") model = next();
        else if (a == "--prompt") prompt = next();
        else if (a == "--steps") steps = std::atoi(next());
        else if (a == "--max-seq") max_seq = std::atoi(next());
        else if (a == "--tpot-steps") tpot_steps = std::atoi(next());
        else if (a == "--mode") mode = std::strcmp(next(), "fast") == 0 ? AF_ENGINE_FAST : AF_ENGINE_EXACT;
        else if (a == "--true-argmax") amode = AF_ARGMAX_TRUE;
        else {
            std::fprintf(stderr, "usage: af_generate --model M.bin --prompt ids.txt [--steps N] [--mode exact|fast] "
                                 "[--max-seq N] [--true-argmax] [--tpot-steps N]\n");
            return 2;
        }
    }
    std::vector<int> ids;
    {
        std::ifstream f(prompt);
        int t;
        while (f >> t) ids.push_back(t);
    }
    if (model.empty() || ids.empty() || steps < 0 || (int)ids.size() + steps + tpot_steps >= max_seq) {
        std::fprintf(stderr, "af_generate: need --model, a non-empty --prompt, and room in the KV cache\n");
        return 2;
    }
    af_engine* e = nullptr;
    af_status st = af_engine_create(model.c_str(), max_seq, mode, amode, &e);
    if (st != AF_OK) return fail("af_engine_create", st);
    // the first step is eager (kernel attributes, workspaces), then one captured
    // step with the position increment serves every later token
    if ((st = af_engine_set_position(e, 0)) != AF_OK || (st = af_engine_inject_token(e, ids[0])) != AF_OK ||
        (st = af_engine_step(e, 0)) != AF_OK || (st = af_engine_capture(e, 1)) != AF_OK ||
        (st = af_engine_set_position(e, 0)) != AF_OK)
        return fail("warm-up", st);
    int tok = 0;
    for (size_t p = 0; p < ids.size(); ++p) {
        if ((st = af_engine_inject_token(e, ids[p])) != AF_OK || (st = af_engine_replay(e, 1)) != AF_OK ||
            (st = af_engine_output_token(e, &tok)) != AF_OK)
            return fail("prompt", st);
    }
    for (int s = 0; s < steps; ++s) {   // greedy: the step's token is the next step's input
        std::printf("%d\n", tok);
        if (s + 1 < steps && ((st = af_engine_replay(e, 1)) != AF_OK || (st = af_engine_output_token(e, &tok)) != AF_OK))
            return fail("greedy step", st);
    }
    if (tpot_steps > 0) {
        cudaStream_t cs = static_cast<cudaStream_t>(af_engine_stream(e));
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, cs);
        if ((st = af_engine_replay(e, tpot_steps)) != AF_OK) return fail("tpot", st);
        cudaEventRecord(b, cs);
        cudaEventSynchronize(b);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, a, b);
        std::printf("tpot_ms %.5f\n", ms / tpot_steps);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
    unsigned faults = 0;
    af_device_faults(&faults, 0);
    af_engine_destroy(e);
    if (faults != 0) {
        std::fprintf(stderr, "af_generate: device fault bits 0x%x\n", faults);
        return 1;
    }
    return 0;
}
