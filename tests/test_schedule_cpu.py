"""The persistent tcgen05 kernel's tile schedule (aotk_gemm_schedule, pure
host arithmetic) without a GPU: every output tile is computed exactly once -
whole, as two N halves, or as all of its K splits - a CTA never receives more
than one tail work item (the K-split reduction stages partials in the A/B
ring, which is only idle after the CTA's last item), and the tail rules hold:
halves for at most SMs/2 leftover tiles, K splits only for at most SMs/4
leftover tiles, at least 128 K blocks and a workspace."""

from __future__ import annotations

import itertools

import pytest

from aot_kernel import capi

SMS = 148


def work_items(sch: dict) -> list[list[tuple]]:
    """Restatement of the device-side work list: per CTA, its items as
    (tile, k_begin, k_end, half) in execution order."""
    out = []
    for cta in range(sch["grid"]):
        items = []
        for r in range(sch["full_rounds"]):
            t = cta + r * sch["grid"]
            if t < sch["split_begin"]:
                items.append((t, 0, sch["kblocks"], -1))
        i = 0
        while True:
            u = cta + i * sch["grid"]
            if u >= sch["units"]:
                break
            if sch["halves"]:
                items.append((sch["split_begin"] + u // 2, 0, sch["kblocks"], u % 2))
            else:
                t = sch["split_begin"] + u // sch["splits"]
                k0 = (u % sch["splits"]) * sch["kb_per_split"]
                items.append((t, k0, min(sch["kblocks"], k0 + sch["kb_per_split"]), -1))
            i += 1
        out.append(items)
    return out


SHAPES = [(m, k, n) for m, k, n in itertools.product(
    (1, 128, 300, 1024, 2048, 4096, 8192, 1280, 2560),
    (64, 1024, 4096, 8192, 14336, 16384),
    (256, 1000, 2048, 4096, 4352, 6144, 14336, 28672))]


@pytest.mark.parametrize("elem_bytes", [2, 1])
@pytest.mark.parametrize("with_ws", [False, True])
def test_every_tile_once_and_one_tail_item_per_cta(elem_bytes, with_ws):
    for M, K, N in SHAPES:
        sch = capi.gemm_schedule(M, N, K, elem_bytes, SMS, with_ws)
        tiles = -(-M // 128) * -(-N // 256)
        assert sch["tiles"] == tiles
        kblocks = -(-K // (128 // elem_bytes))
        assert sch["kblocks"] == kblocks
        assert 1 <= sch["grid"] <= SMS
        cover: dict[int, list] = {}
        for items in work_items(sch):
            tail = [it for it in items if it[0] >= sch["split_begin"]]
            assert len(tail) <= 1, (M, K, N, items)
            if tail:
                assert items[-1] == tail[0]  # the tail item comes last
            for t, k0, k1, h in items:
                cover.setdefault(t, []).append((k0, k1, h))
        assert sorted(cover) == list(range(tiles)), (M, K, N)
        for t, parts in cover.items():
            halves = sorted(h for _, _, h in parts)
            if halves == [0, 1]:
                assert all((k0, k1) == (0, kblocks) for k0, k1, _ in parts)
            else:
                assert all(h == -1 for h in halves)
                ranges = sorted((k0, k1) for k0, k1, _ in parts)
                assert ranges[0][0] == 0 and ranges[-1][1] == kblocks
                assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))  # contiguous, disjoint
        rem = tiles % SMS
        if sch["splits"] > 1:
            assert with_ws and rem * 4 <= SMS and kblocks >= 128 and sch["ws_bytes"] > 0
        else:
            assert sch["ws_bytes"] == 0
        if sch["halves"]:
            assert 0 < 2 * rem <= SMS


def test_tail_rules_on_known_shapes():
    s = capi.gemm_schedule(4096, 4096, 4096, 2, SMS, True)  # 512 tiles: 68 left, K too short
    assert s["halves"] == 1 and s["units"] == 136 and s["ws_bytes"] == 0
    s = capi.gemm_schedule(1280, 4352, 8192, 2, SMS, True)  # 170 tiles: 22 left, 128 K blocks
    assert s["splits"] == 4 and s["units"] == 88 and s["ws_bytes"] > 0
    s = capi.gemm_schedule(1280, 4352, 8192, 2, SMS, False)  # no workspace: halves instead
    assert s["halves"] == 1 and s["splits"] == 1
    s = capi.gemm_schedule(8192, 8192, 8192, 2, SMS, True)  # 2048 tiles: 124 left, run whole
    assert s["halves"] == 0 and s["splits"] == 1 and s["units"] == 0
    s = capi.gemm_schedule(1024, 2048, 2048, 2, SMS, True)  # one partial wave of 64 tiles
    assert s["halves"] == 1 and s["grid"] == 128
    s = capi.gemm_schedule(256, 1024, 16384, 1, SMS, True)  # fp8: 128 K blocks of 128
    assert s["splits"] == 4 and s["kblocks"] == 128


def test_schedule_rejects_bad_arguments():
    with pytest.raises(capi.AotkError):
        capi.gemm_schedule(0, 16, 16, 2, SMS, False)
    with pytest.raises(capi.AotkError):
        capi.gemm_schedule(16, 16, 16, 4, SMS, False)


# ---- aotk_gemm_opt's kernel choice (aotk_gemm_path) ----

@pytest.mark.parametrize("shape,path", [
    ((1, 4096, 28672), "skinny"), ((128, 14336, 4096), "skinny"),
    ((128, 4096, 6144), "skinny"),    # 24 tiles of 256 columns
    ((128, 4096, 28672), "tc"),       # 112 tiles >= 3/4 of 148 SMs: no split-K reduction
    ((96, 4096, 28672), "skinny"),    # M <= 96 stays on the skinny kernel
    ((8192, 8192, 8192), "tc2_wide"), ((16384, 16384, 16384), "tc2_wide"),
    ((8192, 4096, 28672), "tc2_wide"), ((4096, 8192, 57344), "tc2_wide"),
    ((4096, 28672, 8192), "tc2_wide"),  # 256 x 512: 3 rounds + 34 tiles cut into halves; 256 x 256: 7
    ((4096, 4096, 4096), "tc2"),      # 256 pair tiles: 3 rounds + 34 tiles cut into halves
    ((4096, 8192, 7168), "tc"),       # the 8-way TP gate/up: 896 tiles, 8 left for K splits
    ((2048, 2048, 2048), "tc"), ((8192, 2048, 8192), "tc"),
    ((8192, 4100, 8192), "simt"), ((8192, 8192, 8190), "simt")], ids=str)
def test_gemm_path_choices(shape, path):
    M, K, N = shape
    assert capi.gemm_path(M, N, K, SMS) == path


def test_gemm_path_without_workspace_keeps_the_pair_kernel():
    """The pair kernels need no scratch: where one is chosen with a workspace
    the same one is chosen without (only the 1-CTA kernel's tail gets
    slower), so aotk_gemm_opt_workspace_size may report 0 for those shapes."""
    seen = set()
    for M, K, N in itertools.product((256, 1000, 2048, 4096, 8192), (4096, 8192, 14336),
                                     (1024, 4096, 6144, 14336, 28672)):
        p = capi.gemm_path(M, N, K, SMS, True)
        seen.add(p)
        if p != "tc":
            assert capi.gemm_path(M, N, K, SMS, False) == p, (M, K, N)
    assert {"tc", "tc2", "tc2_wide"} <= seen


def test_gemm_path_rejects_bad_arguments():
    with pytest.raises(capi.AotkError):
        capi.gemm_path(0, 8, 8, SMS)

