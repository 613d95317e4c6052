"""Tile / pipeline configuration of the tcgen05 GEMM + epilogue kernel."""

from __future__ import annotations

NUM_SMS_B200 = 148


PAIR_MIN_ROWS = 1024      # stacked rows from which an SM pair owns 256-row tiles


def choose_gemm_config(sk, override: dict, batch: int = 1, allow_pair: bool = True) -> dict:
    """Pick the CTA tile for C[M, N] = A[M, K] @ B[K, N] (+ epilogue).

    One CTA owns a BM x BN output tile with its fp32 accumulator in TMEM;
    BK = 64 bf16 = one 128-byte swizzle row.  BN is chosen to balance the
    persistent tile loop over the SMs.  With enough rows (``pair``), a
    cluster of two CTAs owns a 256 x BN tile (tcgen05.mma.cta_group::2,
    molten/gemm2_sm100.cuh), each staging half of A's rows and half of B's
    columns.
    """
    o = {k: v for k, v in dict(override or {}).items() if k != "prologue"}
    M, N, K = sk.m, sk.n, sk.k
    pair = bool(o.get("pair", batch * M >= PAIR_MIN_ROWS)) and allow_pair
    if pair:
        return _pair_config(M, N, batch, o)
    bm = o.get("bm", 128)
    bk = o.get("bk", 64)
    if "bn" in o:
        bn = o["bn"]
    else:
        best = None
        for cand in (256, 192, 128, 64):
            if N % cand and cand != 64:
                continue
            tiles = batch * -(-M // bm) * -(-N // cand)
            waves = -(-tiles // NUM_SMS_B200)
            eff = tiles / (waves * NUM_SMS_B200)
            if batch * M <= 2 * bm:
                # few row blocks: the GEMM streams B, so fill the SMs first
                # (measured, 64 x 4096 x 14336: BN 128 31 us, 256 44 us, 64 46 us)
                key = (-eff, -cand)
            else:
                key = (-(eff * cand / 256 ** 0.25), -cand)
            if best is None or key < best[0]:
                best = (key, cand)
        bn = best[1]
    stage_bytes = (bm * bk + bk * bn) * 2
    stages = o.get("stages") or max(2, min(8, (200 * 1024) // stage_bytes))
    smem = stages * stage_bytes + (2 * stages + 5) * 8 + 16 + 1024
    if smem > 232448:
        raise ValueError(f"GEMM tile needs {smem} bytes of shared memory")
    group_m = o.get("group_m", 16)
    return {"bm": bm, "bn": bn, "bk": bk, "stages": stages, "group_m": group_m,
            "epi_warps": 4, "threads": 256, "smem_bytes": smem, "pair": False}


def _pair_config(M: int, N: int, batch: int, o: dict) -> dict:
    """SM-pair tiles: 256 x BN per cluster of 2 CTAs, BN in {256, 128}
    (each CTA stages BN/2 columns of B), balanced over the 74 pairs."""
    pairs = NUM_SMS_B200 // 2
    if "bn" in o:
        bn = o["bn"]
        if bn not in (128, 256):
            raise ValueError("SM-pair GEMM tiles have BN 128 or 256")
    else:
        best = None
        for cand in (256, 128):
            tiles = batch * -(-M // 256) * -(-N // cand)
            waves = -(-tiles // pairs)
            eff = tiles / (waves * pairs)
            key = (-(eff * cand / 256 ** 0.25), -cand)
            if best is None or key < best[0]:
                best = (key, cand)
        bn = best[1]
    stage_bytes = (128 * 64 + 64 * (bn // 2)) * 2        # per CTA
    stages = o.get("stages") or max(2, min(8, (232448 - 2048) // stage_bytes))
    smem = stages * stage_bytes + (2 * stages + 5) * 8 + 16 + 1024
    if smem > 232448:
        raise ValueError(f"GEMM tile needs {smem} bytes of shared memory")
    return {"bm": 256, "bn": bn, "bk": 64, "stages": stages, "group_m": o.get("group_m", 16),
            "epi_warps": 4, "threads": 256, "smem_bytes": smem, "pair": True}
