"""Generate tests/golden/bin_layout_tiny.json: the block offsets that the
REFERENCE's own weight loader (include/memory/weight_loader.h) arrives at when
it walks a tiny random-init file in src/core/engine.cu:103-147's order.

Needs the reference checkout (environment variable REF) and g++; run it
where both exist.  The walker below is this project's code: it includes the
reference header and calls its WeightLoader::next<T>() with engine.cu's sizes.
"""
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from atomflow_b200.weights_bin import ModelShape, write_synthetic_bin  # noqa: E402

REF = os.environ.get("REF") or sys.exit("set REF=<reference checkout>")
SHAPE = ModelShape(dim=256, ffn=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab=1000, max_seq_len=64)

WALKER = r'''
#include <cstdio>
#include "memory/weight_loader.h"
int main(int argc, char** argv) {
    WeightLoader L(argv[1]);
    const AtomHeader& h = L.header;
    const size_t D = h.dim, F = h.hidden_dim, V = h.vocab_size, GS = h.group_size;
    const size_t QKV = (size_t)(h.n_heads + 2 * h.n_kv_heads) * (h.dim / h.n_heads);
    std::printf("{\"header\": [%d, %d, %d, %d, %d, %d, %d, %d, %d], \"offsets\": [",
                h.version, h.group_size, h.dim, h.hidden_dim, h.n_layers, h.n_heads, h.n_kv_heads,
                h.vocab_size, h.max_seq_len);
    auto mark = [&](bool last = false) { std::printf("%zu%s", L.current_offset(), last ? "" : ", "); };
    mark();
    L.next<float>(V * D); mark();
    const size_t lin[5][2] = {{QKV, D}, {D, D}, {F, D}, {F, D}, {D, F}};
    for (int i = 0; i < h.n_layers; ++i) {
        L.next<float>(D); mark();
        L.next<float>(D); mark();
        for (auto& nk : lin) {
            L.next<uint8_t>(nk[0] * nk[1]); mark();
            L.next<uint16_t>(nk[0] * (nk[1] / GS)); mark();
        }
    }
    L.next<float>(D); mark();
    L.next<uint16_t>(V * D); mark(true);
    std::printf("], \"file_size\": %zu}\n", L.file_size());
    return 0;
}
'''

with tempfile.TemporaryDirectory() as td:
    src, exe, binf = Path(td) / "walk.cpp", Path(td) / "walk", Path(td) / "tiny.bin"
    src.write_text(WALKER)
    subprocess.check_call(["g++", "-O1", "-std=c++17", f"-I{REF}/include", "-o", str(exe), str(src)])
    write_synthetic_bin(binf, SHAPE, seed=3)
    out = json.loads(subprocess.check_output([str(exe), str(binf)]))
out["shape"] = SHAPE.__dict__
(Path(__file__).parent / "bin_layout_tiny.json").write_text(json.dumps(out, indent=1) + "\n")
print("offsets:", len(out["offsets"]), "file_size:", out["file_size"])
