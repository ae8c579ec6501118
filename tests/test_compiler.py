"""The plugin's StableHLO compiler without a GPU (b200_compile_report): parsing, pattern matching,
fusion planning, NVRTC compilation of generated kernels, and compile-time errors, which name the
unsupported op like the reference's lowering does (src/jam/lower.mm:309)."""
import ctypes
import os

import pytest

from pjrt_b200 import configs
from pjrt_b200.shlo import Builder


def report(lib_path, text, nprocs=1, nvrtc=1):
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(1 << 20)
    t = text.encode()
    rc = lib.b200_compile_report(t, len(t), nprocs, nvrtc, buf, len(buf))
    return rc, buf.value.decode()


@pytest.mark.parametrize("causal", [False, True])
def test_attention_chain_becomes_one_fused_step(lib_path, causal):
    p = configs.attention_program(B=4, H=16, S=1024, causal=causal, with_inputs=False)
    rc, rep = report(lib_path, p.text)
    assert rc == 0, rep
    steps = [l for l in rep.splitlines() if l.startswith("  [")]
    assert len(steps) == 1 and "attention" in steps[0] and (("causal" in steps[0]) == causal), rep


def test_attention_unfused_when_disabled(lib_path, monkeypatch):
    monkeypatch.setenv("B200_NO_FLASH", "1")
    p = configs.attention_program(B=1, H=2, S=256, causal=True, with_inputs=False)
    rc, rep = report(lib_path, p.text)
    assert rc == 0, rep
    assert "attention" not in rep and rep.count("gemm") == 2 and ("reduce" in rep or "row" in rep)


def test_mlp_step_compiles_with_generated_kernels(lib_path):
    rc, rep = report(lib_path, configs.mlp_program(with_inputs=False).text)
    assert rc == 0, rep
    assert rep.count("gemm") == 5 and "reduce" in rep and "loop" in rep


def test_gemm_and_batched_gemm_plans(lib_path):
    rc, rep = report(lib_path, configs.gemm_program(1024, 1024, 1024, with_inputs=False).text)
    assert rc == 0 and "gemm b1 1024x1024x1024" in rep, rep
    rc, rep = report(lib_path, configs.gemm_program(2048, 2048, 2048, batch=16, with_inputs=False).text)
    assert rc == 0 and "gemm b16 2048x2048x2048" in rep, rep


def test_dot_reads_mn_major_operands_in_place(lib_path):
    """x @ W with W [K, N] and x^T @ dy read their operands where they lie (no transpose step)."""
    b = Builder("jit_mn")
    x = b.arg((512, 256), "bf16")
    w = b.arg((256, 384), "bf16")
    dy = b.arg((512, 384), "bf16")
    y = b.dot_general(x, w, contract=([1], [0]), out_dtype="f32")
    dw = b.dot_general(x, dy, contract=([0], [0]), out_dtype="f32")
    rc, rep = report(lib_path, b.text([y, dw]))
    assert rc == 0, rep
    assert "transpose" not in rep and "gemm b1 512x384x256 kn" in rep and "gemm b1 256x384x512 mn" in rep, rep


@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_f32_dot_operand_is_stored_narrow_only_for_16bit_results(lib_path, out):
    """An f32 operand whose dots have bf16 partners and bf16 results is stored rounded and read in
    place by the tensor cores; with f32 results the dots are f32-accurate split products that read
    the f32 value in place."""
    b = Builder("jit_cot")
    x = b.arg((256, 96), "bf16")
    w = b.arg((1001, 96), "bf16")
    z = b.arg((256, 1001), "f32")
    g = b.exp(z) - z
    dx = b.dot_general(g, w, contract=([1], [0]), out_dtype=out)
    dw = b.dot_general(g, x, contract=([0], [0]), out_dtype=out)
    rc, rep = report(lib_path, b.text([dx, dw]))
    assert rc == 0, rep
    assert "transpose" not in rep and rep.count("gemm") == 2 and "loop" in rep, rep
    assert (rep.count("f32-split") == 2) == (out == "f32"), rep


def test_large_f32_dots_use_the_split_tensor_core_product(lib_path):
    rc, rep = report(lib_path, configs.gemm_program(1024, 1024, 1024, dtype="f32", with_inputs=False).text)
    assert rc == 0 and "f32-split" in rep, rep
    rc, rep = report(lib_path, configs.mlp_program(with_inputs=False).text)   # [128,784] x [784,512]: small
    assert rc == 0 and "f32-split" not in rep and "f32-simt" in rep, rep


def test_psum_is_identity_on_one_rank_and_a_collective_on_many(lib_path):
    p = configs.psum_program(1024, 2, with_inputs=False)
    rc, rep = report(lib_path, p.text, nprocs=1)
    assert rc == 0 and "all_reduce" not in rep, rep
    rc, rep = report(lib_path, p.text, nprocs=2)
    assert rc == 0 and "all_reduce tensor<1024xf32>" in rep, rep


def test_unsupported_op_fails_at_compile_time_with_its_name(lib_path):
    text = """
module @m {
  func.func public @main(%arg0: tensor<8xf32>) -> (tensor<8xf32>) {
    %0 = stablehlo.fft %arg0, type = FFT, length = [8] : (tensor<8xf32>) -> tensor<8xf32>
    return %0 : tensor<8xf32>
  }
}
"""
    rc, rep = report(lib_path, text)
    assert rc == 1 and "fft" in rep, rep


def test_all_gather_only_along_dim0(lib_path):
    b = Builder("jit_ag", num_partitions=2)
    x = b.arg((4, 6), "f32")
    y = b.all_gather(x, 2, dim=1)
    rc, rep = report(lib_path, b.text([y]), nprocs=2)
    assert rc == 1 and "dim 0" in rep, rep


def test_malformed_text_is_a_compile_error(lib_path):
    rc, rep = report(lib_path, "module @m { func.func public @main(%arg0: tensor<4xf32>) -> ")
    assert rc == 1 and rep.startswith("error:"), rep
    rc, rep = report(lib_path, "")
    assert rc == 1


def test_generated_kernels_compile_with_nvrtc_for_sm100a(lib_path):
    """Elementwise / broadcast / convert / compare / select / iota / reduce chains -> NVRTC."""
    b = Builder("jit_mix")
    x = b.arg((64, 96), "bf16")
    y = b.arg((96,), "f32")
    xf = b.convert(x, "f32")
    z = b.tanh(xf * 0.5 + y) - b.exp(b.sqrt(b.maximum(xf, 0.0)))
    m = b.compare(b.iota((64, 96), 0), b.iota((64, 96), 1), "LT")
    w = b.select(m, z, b.const(0.0, "f32", (64, 96)))
    r1 = b.sum(w, 1)
    r0 = b.max(w, 0)
    rc, rep = report(lib_path, b.text([b.convert(w, "bf16"), r1, r0]))
    assert rc == 0, rep


def test_small_independent_loops_share_one_launch(lib_path):
    """Updates of several small parameters (no data flow between them) become one merged kernel
    whose CTAs are dispatched to each update by range; a dependent one is not merged."""
    b = Builder("jit_small_updates")
    ps = [b.arg((n,), "f32") for n in (768, 2304, 96)]
    gs = [b.arg((n,), "f32") for n in (768, 2304, 96)]
    outs = [p - 0.1 * g for p, g in zip(ps, gs)]
    outs.append(b.sum(outs[0], [0]) + 1.0)          # reads an update: after the merged kernel
    rc, rep = report(lib_path, b.text(outs))
    assert rc == 0, rep
    assert "loops x3" in rep, rep


def _one_op(body, ins, out):
    sig = ", ".join(f"%arg{i}: {t}" for i, t in enumerate(ins))
    return f"module @m {{\n  func.func public @main({sig}) -> ({out}) {{\n{body}\n    return %0 : {out}\n  }}\n}}\n"


A, Bt, C = "tensor<8x128xf32>", "tensor<8x64xf32>", "tensor<128x8xf32>"
MALFORMED = [
    ("missing operand", _one_op(f"    %0 = stablehlo.exponential  : {A}", [A], A), "expects 1 operand"),
    ("operand type stated wrongly", _one_op(f"    %0 = stablehlo.add %arg0, %arg1 : {A}", [A, Bt], A), "operand 1 of stablehlo.add is"),
    ("binary shapes differ", _one_op(f"    %0 = stablehlo.add %arg0, %arg1 : ({A}, {Bt}) -> {A}", [A, Bt], A), "differs from the result"),
    ("slice out of range", _one_op(f"    %0 = stablehlo.slice %arg0 [0:8, 100:164] : ({A}) -> {Bt}", [A], Bt), "slice bounds"),
    ("broadcast dims", _one_op(f"    %0 = stablehlo.broadcast_in_dim %arg0, dims = [0, 2] : ({A}) -> {A}", [A], A), "broadcast"),
    ("not a permutation", _one_op(f"    %0 = stablehlo.transpose %arg0, dims = [0, 0] : ({A}) -> {C}", [A], C), "permutation"),
    ("reshape count", _one_op(f"    %0 = stablehlo.reshape %arg0 : ({A}) -> {Bt}", [A], Bt), "element count"),
    ("dot contracting sizes", _one_op(f"    %0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : ({A}, {Bt}) -> tensor<8x64xf32>",
                                      [A, Bt], "tensor<8x64xf32>"), "contracting dimensions differ"),
    ("dynamic slice size", _one_op(f"    %0 = stablehlo.dynamic_slice %arg0, %arg1, %arg1, sizes = [16, 64] : ({A}, tensor<i32>, tensor<i32>) -> tensor<16x64xf32>",
                                   [A, "tensor<i32>"], "tensor<16x64xf32>"), "slice size out of range"),
]


@pytest.mark.parametrize("what,text,msg", MALFORMED, ids=[m[0] for m in MALFORMED])
def test_malformed_programs_are_rejected_at_compile_time(lib_path, what, text, msg):
    """Programs MLIR's verifiers would reject fail to compile (never become out-of-bounds kernels)."""
    rc, rep = report(lib_path, text, nvrtc=0)
    assert rc == 1 and msg in rep, rep


_FUZZ_CHILD = r'''
import ctypes, json, sys
lib = ctypes.CDLL(sys.argv[1])
buf = ctypes.create_string_buffer(1 << 23)
for t in json.loads(sys.stdin.read()):
    b = t.encode()
    assert lib.b200_compile_report(b, len(b), 1, 0, buf, len(buf)) in (0, 1)
print("ok")
'''


def test_mutated_programs_never_crash_the_compiler(lib_path):
    """Seeded token-level mutations of real programs (dropped, duplicated and altered tokens):
    parse + verify + lower end in a plan or an error, never a crash, in a child process."""
    import json
    import random
    import re
    import subprocess
    import sys
    progs = [configs.mlp_program(with_inputs=False).text,
             configs.attention_program(B=1, H=2, S=256, causal=True, with_inputs=False).text,
             configs.gpt2_program(layers=1, d=64, heads=2, mlp=128, vocab=96, seq=64, batch=2, with_inputs=False).text]
    rng = random.Random(2024)
    tok = re.compile(r"\s+|[^\s]+")
    items = []
    for _ in range(300):
        toks = tok.findall(rng.choice(progs))
        for _ in range(rng.randint(1, 3)):
            k = rng.randrange(len(toks))
            r = rng.random()
            if r < 0.4:
                toks[k] = ""
            elif r < 0.7:
                toks[k] = toks[rng.randrange(len(toks))]
            else:
                toks[k] = re.sub(r"\d+", lambda m: str(rng.choice([0, 1, 7, 65536, 2 ** 31])), toks[k])
        items.append("".join(toks))
    r = subprocess.run([sys.executable, "-c", _FUZZ_CHILD, lib_path], input=json.dumps(items).encode(),
                       capture_output=True, timeout=600)
    assert r.returncode == 0 and b"ok" in r.stdout, r.stderr[-2000:]


ONE_RANK = {
    "all_to_all": '"stablehlo.all_to_all"(%arg0) <{concat_dimension = 0 : i64, replica_groups = dense<[[0]]> : tensor<1x1xi64>, split_count = 1 : i64, split_dimension = 0 : i64}>',
    "collective_broadcast": '"stablehlo.collective_broadcast"(%arg0) <{replica_groups = dense<[[0]]> : tensor<1x1xi64>}>',
    "collective_permute": '"stablehlo.collective_permute"(%arg0) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, source_target_pairs = dense<[[0, 0]]> : tensor<1x2xi64>}>',
}


@pytest.mark.parametrize("name", sorted(ONE_RANK))
def test_other_collectives_are_identities_at_one_process(lib_path, name):
    """all_to_all / collective_broadcast / collective_permute at one process return their operand
    (the reference binds them to it, src/jam/ops/collectives.mm:16-29); across processes they are
    a compile error naming the op."""
    text = _one_op(f"    %0 = {ONE_RANK[name]} : ({A}) -> {A}", [A], A)
    rc, rep = report(lib_path, text, nvrtc=0)
    assert rc == 0 and "kernel" not in rep and "collective" not in rep.split("\n", 1)[-1], rep
    rc, rep = report(lib_path, text, nprocs=2, nvrtc=0)
    assert rc == 1 and name in rep and "across processes" in rep, rep


def test_collective_permute_without_self_pair_is_refused_at_one_process(lib_path):
    text = _one_op(f"    %0 = " + ONE_RANK["collective_permute"].replace("[[0, 0]]", "[[1, 0]]") + f" : ({A}) -> {A}", [A], A)
    rc, rep = report(lib_path, text, nvrtc=0)
    assert rc == 1 and "(0, 0) pair" in rep, rep


@pytest.mark.parametrize("groups,ok", [("[[0, 1]]", True), ("[[1, 0]]", False), ("[[0], [1]]", False)])
def test_collectives_across_processes_need_one_world_group(lib_path, groups, ok):
    """The NCCL communicator spans all ranks in rank order: a program whose replica groups split
    the ranks or reorder them is refused at compile time instead of running world-wide."""
    p = configs.psum_program(1024, 2, with_inputs=False)
    n = groups.count("[") - 1
    text = p.text.replace("dense<[[0, 1]]> : tensor<1x2xi64>", f"dense<{groups}> : tensor<{n}x{2 // n}xi64>")
    assert text != p.text or groups == "[[0, 1]]"
    rc, rep = report(lib_path, text, nprocs=2)
    if ok:
        assert rc == 0 and "all_reduce" in rep, rep
    else:
        assert rc == 1 and "replica_groups" in rep, rep


def test_small_all_reduces_are_issued_as_nccl_groups(lib_path, monkeypatch):
    """Across processes, the DP step's small gradient all-reduces (<= 256 KiB) are held back and
    issued together as NCCL groups; large ones keep their hoisted places."""
    monkeypatch.setenv("B200_NO_PACK", "1")
    p = configs.gpt2_program(batch=2, world=2, layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64, with_inputs=False)
    rc, rep = report(lib_path, p.text, nprocs=2)
    assert rc == 0, rep
    colls = [l for l in rep.splitlines() if "all_reduce" in l]
    grouped = [l for l in colls if "[group" in l]
    assert len(colls) > 10 and len(grouped) >= len(colls) // 2, rep
    rc, rep1 = report(lib_path, p.text, nprocs=1)
    assert rc == 0 and "[group" not in rep1


def _options_report(lib_path, data):
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(4096)
    rc = lib.b200_compile_options_report(data, len(data), buf, len(buf))
    return rc, buf.value.decode()


def test_compile_options_proto_fields_decode_like_the_protobuf_library(lib_path):
    """PJRT_Client_Compile's compile_options bytes (xla.CompileOptionsProto) as the protobuf library
    writes them (tests/golden/make_compile_options.py): the plugin reads num_replicas /
    num_partitions and the device assignment, and skips every other field."""
    import json
    with open(os.path.join(os.path.dirname(__file__), "golden", "compile_options.json")) as f:
        cases = json.load(f)
    assert len(cases) >= 4
    for c in cases:
        rc, rep = _options_report(lib_path, bytes.fromhex(c["hex"]))
        assert rc == 0 and rep == c["expect"], (c["name"], rep)


def test_malformed_compile_options_are_rejected(lib_path):
    import json
    with open(os.path.join(os.path.dirname(__file__), "golden", "compile_options.json")) as f:
        good = bytes.fromhex(next(c for c in json.load(f) if c["name"] == "shard_map_8")["hex"])
    for cut in range(1, len(good)):
        rc, rep = _options_report(lib_path, good[:cut])
        assert rc in (0, 1) and (rc == 0 or rep.startswith("error:"))
    rc, rep = _options_report(lib_path, b"\x1a\xff\xff\xff\xff\x0f")     # field 3 claiming 4 GB
    assert rc == 1 and "past the end" in rep, rep
    rc, rep = _options_report(lib_path, b"\x1f")                          # wire type 7
    assert rc == 1, rep


# ---------------------------------------------------------------------------- buffer donation
def _donated_lines(rep):
    return {int(l.split()[2]): l for l in rep.splitlines() if l.startswith("  donated argument")}


def test_donated_optimizer_state_is_updated_in_place(lib_path):
    """jax.jit(step, donate_argnums=...) marks each donated parameter / moment with
    tf.aliasing_output; the AdamW update kernels read them only at the element they write, after
    every other reader, so every result goes into its argument's buffer (also across processes)."""
    for world in (1, 2):
        p = configs.gpt2_program(batch=2, world=world, layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64,
                                 with_inputs=False, donate=True)
        rc, rep = report(lib_path, p.text, nprocs=world)
        assert rc == 0, rep
        lines = _donated_lines(rep)
        n_state = 3 * p.meta["n_tensors"]
        assert len(lines) == n_state and all("written in place" in l for l in lines.values()), rep


def _alias_program(make, aliases, donors=()):
    b = Builder("jit_alias")
    x, y = b.arg((64, 128), "f32"), b.arg((64, 128), "f32")
    return b.text(make(b, x, y), aliases=aliases, donors=donors)


def test_donation_in_place_only_where_it_is_safe(lib_path):
    # elementwise: in place
    rc, rep = report(lib_path, _alias_program(lambda b, x, y: [x * 2.0 + y], {0: 0}))
    assert rc == 0 and "written in place" in _donated_lines(rep)[0], rep
    # the result is the argument itself: in place (the output copy becomes a no-op)
    rc, rep = report(lib_path, _alias_program(lambda b, x, y: [x, y + 1.0], {0: 0}))
    assert rc == 0 and "written in place" in _donated_lines(rep)[0], rep
    # a row kernel (softmax over the rows of the donated argument): a fresh buffer
    def softmax(b, x, y):
        e = b.exp(x - b.broadcast_to(b.max(x, -1, keepdims=True), x.shape))
        return [e / b.broadcast_to(b.sum(e, -1, keepdims=True), x.shape)]
    rc, rep = report(lib_path, _alias_program(softmax, {0: 0}))
    assert rc == 0 and "fresh buffer" in _donated_lines(rep)[0], rep
    # the donated argument read at another element (its transpose): a fresh buffer
    b = Builder("jit_alias_t")
    x, y = b.arg((64, 64), "f32"), b.arg((64, 64), "f32")
    rc, rep = report(lib_path, b.text([b.transpose(x, (1, 0)) + y], aliases={0: 0}))
    assert rc == 0 and "fresh buffer" in _donated_lines(rep)[0], rep
    # a buffer donor without an alias is listed, no result is tied to it
    rc, rep = report(lib_path, _alias_program(lambda b, x, y: [x + y], {}, donors=(1,)))
    assert rc == 0 and _donated_lines(rep)[1].strip() == "donated argument 1", rep


@pytest.mark.parametrize("aliases,err", [({0: 1}, "has 1 results"), ({0: 0, 1: 0}, "of two arguments")])
def test_bad_aliasing_is_a_compile_error(lib_path, aliases, err):
    rc, rep = report(lib_path, _alias_program(lambda b, x, y: [x + y], aliases))
    assert rc == 1 and err in rep, rep


def test_alias_between_different_types_is_a_compile_error(lib_path):
    b = Builder("jit_alias")
    x = b.arg((64, 128), "f32")
    rc, rep = report(lib_path, b.text([b.convert(x, "bf16")], aliases={0: 0}))
    assert rc == 1 and "cannot alias result 0" in rep, rep


def test_cross_entropy_backward_joins_its_forward_row_walk(lib_path, monkeypatch):
    """The mean cross-entropy sums the per-row losses between the forward row kernel (max, sum of
    exponentials, picked logit) and the backward (softmax - one-hot): that sum is held back behind
    the row group, so the backward becomes a second walk of the same kernel instead of a separate
    pass over the logits."""
    p = configs.gpt2_program(batch=2, world=1, layers=1, d=64, heads=2, mlp=128, vocab=1000, seq=64, with_inputs=False)
    rc, rep = report(lib_path, p.text)
    assert rc == 0, rep
    over_logits = [l for l in rep.splitlines() if "tensor<128x1000xf32>" in l]
    assert len(over_logits) == 1 and "row" in over_logits[0] and "x4" in over_logits[0], rep
    monkeypatch.setenv("B200_NO_DEFER", "1")
    rc, rep = report(lib_path, p.text)
    assert rc == 0 and len([l for l in rep.splitlines() if "tensor<128x1000xf32>" in l]) == 2, rep


@pytest.mark.parametrize("bucket", ["", "all"])
def test_grouped_all_reduces_are_packed_into_one_bucket(lib_path, monkeypatch, bucket):
    """The all-reduces of one NCCL group (one type, one reduction) become a single all-reduce over a
    bucket that their inputs and outputs live in; with B200_COLL_BUCKET=all every gradient of the
    step is held for it.  Every gradient is still reduced exactly once: the packed members' bytes
    (each rounded up to 256) add up to the buckets."""
    import re
    if bucket:
        monkeypatch.setenv("B200_COLL_BUCKET", bucket)
    p = configs.gpt2_program(batch=2, world=2, layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64, with_inputs=False)
    rc, rep = report(lib_path, p.text, nprocs=2)
    assert rc == 0, rep
    colls = [l for l in rep.splitlines() if "all_reduce" in l]
    packed = [l for l in colls if "packed" in l]
    members = sum(int(re.search(r"packed x(\d+)", l).group(1)) for l in packed)
    assert packed and members + len(colls) - len(packed) == 29, rep   # 28 gradients + the loss
    if bucket == "all":
        assert len(colls) <= 8, rep


def test_sibling_column_reductions_stay_merged_when_rounded_for_all_reduce(lib_path, monkeypatch):
    """Across processes each LayerNorm's two parameter gradients (column sums over the same rows) are
    rounded to bf16 for their all_reduce.  The roundings wait behind the open column-reduction group,
    so the second sum still joins the first one's kernel (one read of the shared dy) and the two
    roundings share a launch; without the hold-back every sum runs alone."""
    p = configs.gpt2_program(batch=2, world=2, layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64, with_inputs=False)
    rc, rep = report(lib_path, p.text, nprocs=2)
    assert rc == 0, rep
    sums = [l for l in rep.splitlines() if "-> tensor<64xf32>" in l and "all_reduce" not in l]
    assert len(sums) == 5 and all("reduce x2" in l for l in sums), rep
    monkeypatch.setenv("B200_NO_DEFER", "1")
    rc, rep = report(lib_path, p.text, nprocs=2)
    sums = [l for l in rep.splitlines() if "-> tensor<64xf32>" in l and "all_reduce" not in l]
    assert rc == 0 and len(sums) == 10 and not any("reduce x2" in l for l in sums), rep
