"""Host logic of libtpsa.so on CPU: exports, attribute gates, tile schedule.

No kernel runs here; tpsa_make_plan / tpsa_plan_item / tpsa_plan_tile are
pure host functions (given an explicit SM count) built from the same
header the kernel uses (csrc/tpsa_schedule.h).
"""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import triangle_oracle as o

ROOT = Path(__file__).resolve().parents[1]
SM = 148


def test_library_exports_every_declared_symbol(tm):
    header = (ROOT / "include" / "tpsa.h").read_text()
    declared = set(re.findall(r"TPSA_API\s+[\w\s\*]+?\b(tpsa_\w+)\s*\(", header))
    assert declared == set(tm._native.EXPORTED_SYMBOLS)
    nm = subprocess.run(["nm", "-D", "--defined-only", str(tm._native.LIB_PATH)], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tpsa_\w+)", nm))
    assert declared <= exported
    lib = tm._native.lib()
    for name in declared:
        assert hasattr(lib, name)
    define = re.search(r"#define TPSA_ABI_VERSION (\d+)", header)
    assert define and lib.tpsa_abi_version() == int(define.group(1)) == tm._native.ABI_VERSION


def test_adapter_library_is_built(tm):
    assert tm._native.ADAPTER_PATH.exists()
    nm = subprocess.run(["nm", "-D", "--undefined-only", str(tm._native.ADAPTER_PATH)],
                        capture_output=True, text=True, check=True).stdout
    assert "tpsa_paged_attention" in nm and "tpsa_workspace_size" in nm


@pytest.mark.parametrize("args,msg", [
    ((10, 1, 10, 10), "query_start + Tq == seq_len"),
    ((10, 0, 10, 9), "invalid query_start/seq_len/prompt_len/scale"),
    ((0, 0, 0, 0), "invalid query_start/seq_len/prompt_len/scale"),
    ((10, -1, 9, 10), "invalid query_start/seq_len/prompt_len/scale"),
    ((10, 0, 10, 2 ** 33), "UINT32_MAX"),
])
def test_attribute_gates(tm, args, msg):
    with pytest.raises(tm.TpsaError, match=re.escape(msg)):
        tm._native.make_plan(*args, kv_heads=8, sm_count=SM)


def test_scale_and_head_gates(tm):
    for scale in (0.0, -1.0, float("inf"), float("nan")):
        with pytest.raises(tm.TpsaError):
            tm._native.make_plan(10, 0, 10, 10, 8, SM, scale)
    for kvh in (0, 3, 16):
        with pytest.raises(tm.TpsaError, match="kv_heads"):
            tm._native.make_plan(10, 0, 10, 10, kvh, SM)


def test_wait_probe_limit_gate(tm):
    """The test hook takes 0 (disarm) or a limit in [1 us, 100 ms]; arming
    and disarming touch no device."""
    for bad in (1, 999, 100_000_001, 2 ** 32 - 1):
        with pytest.raises(tm.TpsaError, match="probe limit"):
            tm._native.debug_wait_probe(bad)
    tm._native.debug_wait_probe(200_000)
    tm._native.debug_wait_probe(0)


CASES = [
    (0, 1, 1, 1024), (0, 5, 5, 2048), (250, 5, 255, 2048), (519, 4, 523, 2048), (500, 65, 565, 2048),
    (766, 35, 801, 2048), (894, 4, 898, 1024), (1023, 1, 1024, 1024), (0, 4096, 4096, 4096),
    (0, 8192, 8192, 8192), (2048, 512, 2560, 2869), (2560, 309, 2869, 2869), (6272, 2048, 8320, 8320),
    (24576, 8192, 32768, 32768), (0, 600, 600, 600), (8127, 65, 8192, 16384), (3000, 1096, 4096, 4096),
    (57344, 8192, 65536, 65536),
]


@pytest.mark.parametrize("q0,tq,seq,prompt", CASES)
def test_tile_schedule_covers_exact_key_sets(tm, q0, tq, seq, prompt):
    """Per block: each 64-key half of a tile is page-contained, the tiles
    cover every visible key, and they load no key outside the 64-rounded
    union of the block's key sets."""
    plan = tm._native.make_plan(tq, q0, seq, prompt, 8, SM)
    assert plan.num_blocks == -(-tq // 64)
    for b in range(plan.num_blocks):
        q_lo, q_hi = q0 + 64 * b, min(q0 + 64 * b + 64, seq)
        rows = np.arange(q_lo, q_hi)
        union = np.zeros(seq + 128, dtype=bool)
        t = 0
        loaded = []
        while True:
            try:
                k0, w, masked, up = tm._native.plan_tile(plan, b, t)
            except tm.TpsaError:
                break
            assert w in (64, 80, 128) and k0 % 64 == 0 and up % 64 == 0
            if w == 80:
                # the composite tile of a sparse block: the band's 64-key edge
                # and the first 16 keys of the sink page, always masked
                assert t == 0 and k0 >= 128 and up == 0 and masked
                runs = [(k0, 64), (0, 16)]
            else:
                assert up == k0 + 64
                assert k0 // 128 == (k0 + w - 1) // 128, "tile crosses a page"
                runs = [(k0, w)]
            for h, n in runs:
                assert h + n <= -(-seq // 128) * 128, "tile beyond the block table"
            keys = np.concatenate([np.arange(h, h + n) for h, n in runs])
            vis = o.visible_mask(rows, keys, seq, prompt)
            if not masked:
                assert vis.all(), f"unmasked tile {k0}+{w} hides keys of block {b}"
            loaded.append(keys)
            t += 1
        loaded_keys = np.concatenate(loaded)
        assert len(set(loaded_keys.tolist())) == loaded_keys.size, "a key is loaded twice"
        vis_all = o.visible_mask(rows, np.arange(seq), seq, prompt).any(axis=0)
        union[: seq][vis_all] = True
        assert union[loaded_keys].sum() == vis_all.sum(), "a visible key is not loaded"
        # Nothing beyond 64-key rounding of the needed ranges is loaded.
        needed_grains = set((np.nonzero(vis_all)[0] // 64).tolist())
        assert set((loaded_keys // 64).tolist()) == needed_grains


@pytest.mark.parametrize("q0,tq,seq,prompt", CASES)
def test_items_partition_blocks_heads_and_tiles(tm, q0, tq, seq, prompt):
    for kvh in (8, 2):
        plan = tm._native.make_plan(tq, q0, seq, prompt, kvh, SM)
        seen = {}
        costs = []
        for i in range(plan.total_items):
            it = tm._native.plan_item(plan, i)
            key = (it.block, it.kv_head)
            seen.setdefault(key, []).append((it.split, it.tile_begin, it.tile_end, it.num_splits))
            costs.append(it.tile_end - it.tile_begin)
            assert it.tile_end > it.tile_begin
            assert it.tile_end - it.tile_begin <= max(plan.split_tiles, 7)
        assert set(seen) == {(b, h) for b in range(plan.num_blocks) for h in range(kvh)}
        for (b, _), parts in seen.items():
            parts.sort()
            assert [p[0] for p in parts] == list(range(parts[0][3]))
            assert parts[0][1] == 0
            for a, c in zip(parts, parts[1:]):
                assert a[2] == c[1]
            ntiles = 0
            while True:
                try:
                    tm._native.plan_tile(plan, b, ntiles)
                    ntiles += 1
                except tm.TpsaError:
                    break
            assert parts[-1][2] == ntiles
        assert sum(costs) == plan.total_tiles
        assert plan.grid == min(plan.total_items, SM)  # one CTA per item at a time
        split = any(tm._native.plan_item(plan, i).num_splits > 1 for i in range(plan.tail_items))
        assert plan.workspace_bytes == 2048 + (plan.tail_items * 256 * 130 * 4 if split else 0)
        assert (plan.num_blocks - plan.tail_block0) * kvh * 2 <= 448 or not split


def test_long_tail_blocks_are_split_and_run_first(tm):
    plan = tm._native.make_plan(8192, 24576, 32768, 32768, 8, SM)
    first = tm._native.plan_item(plan, 0)
    assert first.num_splits > 1 and first.block == plan.num_blocks - 1
    longest = max(tm._native.plan_item(plan, i).tile_end - tm._native.plan_item(plan, i).tile_begin
                  for i in range(plan.total_items))
    assert longest <= plan.split_tiles
    assert plan.total_tiles / SM >= longest


@pytest.mark.parametrize("seq, pieces", [(8192, 2), (32768, 5), (65536, 6), (131072, 8)])
def test_tail_split_count_fits_the_ctas(tm, seq, pieces):
    """BASELINE config 3 (8192-row chunk ending an N-token prompt): the 16
    dense-tail (block, head) items are cut into as many pieces as the
    makespan estimate picks for 148 CTAs: at 128K 8 pieces (128 pieces of
    128 tiles, one per CTA, beside an average of 145 tiles per CTA), never
    more pieces than CTAs."""
    plan = tm._native.make_plan(8192, seq - 8192, seq, seq, 8, SM)
    tail_blocks = (plan.num_blocks - plan.tail_block0) * 8
    assert plan.tail_items == tail_blocks * pieces
    assert plan.tail_items <= SM


def test_static_scratch_range_fits_its_array(tm):
    """Every plan the static-scratch entry point documents (query chunks of
    64-16384 rows at the end of prompts of 4K-4M tokens) fits in 24 MiB."""
    worst = 0
    for seq in (4096, 16384, 65536, 262144, 1 << 20, 1 << 22):
        for tq in (64, 128, 256, 1024, 4096, 8192, 16384):
            if tq <= seq:
                worst = max(worst,
                            tm._native.make_plan(tq, seq - tq, seq, seq, 8, SM).workspace_bytes)
    assert worst <= 24 << 20


def test_workspace_is_control_words_without_splits(tm):
    # Intermediate chunk with no dense tail: nothing is split, only the
    # scheduler's control words are needed.
    plan = tm._native.make_plan(2048, 2048, 4096, 8320, 8, SM)
    assert plan.workspace_bytes == 2048 and plan.tail_items == 0


@pytest.mark.parametrize("cu, seq_lens, prompt_lens, message", [
    ([0, 10, 10], [10, 20], [10, 20], "each ragged query length must be positive"),
    ([1, 10], [10], [10], "cu_seqlens_q[0] must be 0"),
    ([0, 30], [20], [20], "seq_lens[i] must cover the request's query rows"),
])
def test_varlen_metadata_gates_on_host(tm, cu, seq_lens, prompt_lens, message):
    """The packed-batch gates run before any device call (reference
    triangle_v2_reference.py:466-475 rejects the same metadata)."""
    import ctypes

    nat = tm._native
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: the metadata gate fails first
    st = nat.lib().tpsa_paged_attention_varlen(fake, fake, fake, fake, fake, len(seq_lens),
                                               nat._int64_array(cu), nat._int64_array(seq_lens),
                                               nat._int64_array(prompt_lens), 8, 1, 0.088, fake,
                                               1 << 20, None)
    assert st == 1  # TPSA_ERR_INVALID_ARGUMENT
    assert message in nat.lib().tpsa_last_error().decode()


def test_adapter_registers_the_reference_schemas(tm):
    """Loading the adapter (no GPU needed) registers the reference's operator
    names and schemas (operator/torch_adapter/triangle_paged_attention_torch.cpp
    :265-297, README.md:34-36 of the reference)."""
    import torch

    tm.load_adapter()
    args = ("(Tensor query, Tensor key_cache, Tensor value_cache, Tensor block_table, "
            "int query_start, int seq_len, int prompt_len, float scale")
    out = ", *, Tensor(a!) out) -> Tensor(a!)"
    assert str(torch.ops.trianglemix.triangle_paged_sparse_attention.out._schema) == (
        "trianglemix::triangle_paged_sparse_attention.out" + args + out)
    assert str(torch.ops._C_ascend.npu_triangle_paged_sparse_attention.default._schema) == (
        "_C_ascend::npu_triangle_paged_sparse_attention" + args + out)
    assert str(torch.ops.trianglemix_reference.triangle_paged_sparse_attention.default._schema) == (
        "trianglemix_reference::triangle_paged_sparse_attention" + args + ") -> Tensor")


def test_estimate_tile_counts_is_this_kernels_plan(tm):
    cfg = tm.TriangleMixConfig(enabled=True, layer_indices=frozenset({1}))
    tri, dense = tm.estimate_tile_counts(8192, cfg)
    assert tri == tm._native.make_plan(8192, 0, 8192, 8192, 8, SM).total_tiles // 8
    assert dense == sum(-(-(64 * (b + 1)) // 128) for b in range(128))
    assert tri < dense
    assert tm.estimate_tile_counts(0, cfg) == (0, 0)
