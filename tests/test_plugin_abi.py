"""Compile-time ABI check of the PufferLib plug-in against the reference's
own type definitions (CPU only: nvcc compiles, nothing runs).

Two translation units are compiled with the reference trainer's build flags
(native/build_native.sh:80-88):

1. the reference's native/src/models.cu (which brings tensor.h and the
   Allocator of kernels.cu), then include/ptcg_puffer.h without the type
   aliases: every member of PrecisionTensor, FloatTensor, AllocEntry,
   Allocator, Encoder, Decoder and Network must sit at the same offset as in
   the header's restated types;
2. models.cu, then the replacement ocean.cu exactly as INTEGRATION.md gives
   it, then the trainer's own calls into the model's exports
   (native/src/pufferlib.cu:1969-1973, 2676-2678) with the trainer's types.

Needs a checkout of the reference: set PTCG_REFERENCE to its root.
"""
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

REF = os.environ.get("PTCG_REFERENCE")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

pytestmark = pytest.mark.skipif(
    not REF or not os.path.exists(os.path.join(REF or "", "native", "src", "models.cu"))
    or not shutil.which(NVCC) and not os.path.exists(NVCC),
    reason="needs PTCG_REFERENCE (a reference checkout) and nvcc")

HEAD = """#include <cstddef>
#include <string>
#include "models.cu"
"""

LAYOUT = HEAD + """#include "ptcg_puffer.h"
#define SAME(T, U, m) static_assert(offsetof(T, m) == offsetof(U, m), #T "." #m)
#define SIZE(T, U) static_assert(sizeof(T) == sizeof(U), "sizeof " #T)
SIZE(PrecisionTensor, PtcgPufTensor); SAME(PrecisionTensor, PtcgPufTensor, data);
SAME(PrecisionTensor, PtcgPufTensor, shape);
SIZE(FloatTensor, PtcgPufTensor); SAME(FloatTensor, PtcgPufTensor, shape);
SIZE(AllocEntry, PtcgPufAllocEntry); SAME(AllocEntry, PtcgPufAllocEntry, data_ptr);
SAME(AllocEntry, PtcgPufAllocEntry, shape); SAME(AllocEntry, PtcgPufAllocEntry, elem_size);
SIZE(Allocator, PtcgPufAllocator); SAME(Allocator, PtcgPufAllocator, regs);
SAME(Allocator, PtcgPufAllocator, num_regs); SAME(Allocator, PtcgPufAllocator, mem);
SAME(Allocator, PtcgPufAllocator, total_elems); SAME(Allocator, PtcgPufAllocator, total_bytes);
#define COMMON(T, U) SAME(T, U, init_weights); SAME(T, U, reg_params); SAME(T, U, reg_train); \\
    SAME(T, U, reg_rollout); SAME(T, U, create_weights); SAME(T, U, free_weights); \\
    SAME(T, U, free_activations)
SIZE(Encoder, PtcgPufEncoder); SAME(Encoder, PtcgPufEncoder, forward);
SAME(Encoder, PtcgPufEncoder, backward); COMMON(Encoder, PtcgPufEncoder);
SAME(Encoder, PtcgPufEncoder, in_dim); SAME(Encoder, PtcgPufEncoder, out_dim);
SAME(Encoder, PtcgPufEncoder, activation_size);
SIZE(Decoder, PtcgPufDecoder); SAME(Decoder, PtcgPufDecoder, forward);
SAME(Decoder, PtcgPufDecoder, backward); COMMON(Decoder, PtcgPufDecoder);
SAME(Decoder, PtcgPufDecoder, hidden_dim); SAME(Decoder, PtcgPufDecoder, output_dim);
SAME(Decoder, PtcgPufDecoder, continuous); SAME(Decoder, PtcgPufDecoder, activation_size);
SIZE(Network, PtcgPufNetwork); SAME(Network, PtcgPufNetwork, forward);
SAME(Network, PtcgPufNetwork, forward_train); SAME(Network, PtcgPufNetwork, backward);
COMMON(Network, PtcgPufNetwork); SAME(Network, PtcgPufNetwork, hidden);
SAME(Network, PtcgPufNetwork, num_layers); SAME(Network, PtcgPufNetwork, horizon);
// the trainer's TrainGraph member 6 (mb_returns) at the offset the plug-in reads
static_assert(offsetof(TrainGraph_probe, mb_returns) == 6 * sizeof(PtcgPufTensor), "mb_returns");
"""

TRAINER_CALLS = """
// the trainer's calls, as native/src/pufferlib.cu makes them
void trainer_calls(PrecisionTensor* v, PrecisionTensor* r, PrecisionTensor* d,
                   PrecisionTensor* imp, PrecisionTensor* obs, PrecisionTensor* adv,
                   void* train_buf, cudaStream_t s) {
    ptcg_puff_advantage(v, r, d, imp, obs, adv, 0.99f, 0.95f, 1.0f, 1.0f, s);
    ptcg_bind_train_graph(train_buf);
    Encoder e{}; Decoder dd{}; Network n{};
    create_custom_encoder("ptcg", &e);
    create_custom_decoder("ptcg", &dd);
    create_custom_network("ptcg", &n);
}
"""


def _train_graph_probe():
    """TrainGraph's first seven members (native/src/pufferlib.cu:116-123),
    named from that file so a reordering there fails the check."""
    src = open(os.path.join(REF, "native", "src", "pufferlib.cu")).read()
    body = re.search(r"struct TrainGraph\s*\{(.*?)\};", src, re.S).group(1)
    names = re.findall(r"PrecisionTensor\s+(\w+)\s*;", body)
    assert names[6] == "mb_returns", names
    return "struct TrainGraph_probe {\n" + "".join(
        f"    PrecisionTensor {n};\n" for n in names) + "};\n"


def _ocean_from_integration():
    txt = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    m = re.search(r"```c\+\+\n(// ocean\.cu.*?)```", txt, re.S)
    assert m, "replacement ocean.cu block not found"
    return m.group(1)


def _compile(tmp_path, name, src):
    p = tmp_path / name
    p.write_text(src)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
           "-DPRECISION_FLOAT", "-DPTCG_NATIVE", "-DOBS_TENSOR_T=FloatTensor", "-DENV_NAME=ptcg",
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(REF, "native", "src"),
           "-c", str(p), "-o", str(tmp_path / (name + ".o"))]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_plugin_types_match_reference_layout(tmp_path):
    src = LAYOUT.replace('#include "ptcg_puffer.h"',
                         '#include "ptcg_puffer.h"\n' + _train_graph_probe())
    _compile(tmp_path, "layout.cu", src)


def test_replacement_ocean_cu_compiles_in_the_trainer(tmp_path):
    _compile(tmp_path, "ocean_tu.cu", HEAD + _ocean_from_integration() + TRAINER_CALLS)
