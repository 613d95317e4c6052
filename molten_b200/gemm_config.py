"""Tile / pipeline configuration of the tcgen05 GEMM + epilogue kernel."""

from __future__ import annotations

NUM_SMS_B200 = 148


PAIR_MIN_ROWS = 1024      # stacked rows from which an SM pair owns 256-row tiles
SK_MAX_PIECES = 10        # most stream-K CTAs that share one output tile


def choose_gemm_config(sk, override: dict, batch: int = 1, allow_pair: bool = True,
                       allow_streamk: bool = True) -> dict:
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
    cfg = {"bm": bm, "bn": bn, "bk": bk, "stages": stages, "group_m": group_m,
           "epi_warps": 4, "threads": 256, "smem_bytes": smem, "pair": False, "streamk": False}
    # few tiles and long K (decode-size M): stream-K spreads the k-blocks of
    # all tiles evenly over the SMs (molten/gemm_sk_sm100.cuh).  Measured
    # (CUDA-graph replay, bf16): 16x8192x1024 (16 tiles) 40.5 -> 20.0 us,
    # 64x14336x4096 (64 tiles) 67.8 -> 42.2 us, 64x4096x4096 (64 tiles)
    # 23.7 -> 23.6 us; with 112-128 tiles it loses (64x4096x14336 27.9 ->
    # 41.1 us: the partial-tile traffic outweighs the SMs it adds), so only
    # up to half the SMs' worth of tiles.  A tile cut into many pieces pays
    # for summing them in one CTA (1x4096x256 over 148 CTAs, 37 pieces:
    # 22.0 -> 26.0 us), so at most SK_MAX_PIECES CTAs per tile (the same
    # shape over 40 CTAs, 10 pieces a tile: 22.1 -> 14.2 us).
    tiles = batch * -(-M // bm) * -(-N // bn)
    kb = -(-K // bk)
    ctas = int(o.get("sk_ctas", min(NUM_SMS_B200, tiles * SK_MAX_PIECES, tiles * kb)))
    auto = tiles <= NUM_SMS_B200 // 2 and tiles * kb >= 2 * ctas and batch * M <= 512
    if o.get("streamk", auto) and allow_streamk:
        # "sk_splits": S > 0 walks split-K units (split-major, so the CTAs
        # running together read the same k-regions of B); 0 walks stream-K
        # ranges (one equal range per CTA)
        splits = min(int(o.get("sk_splits", 0)), kb)         # no empty units
        maxseg = splits if splits > 0 else stream_k_max_segments(tiles, kb, ctas)
        cfg.update(streamk=True, sk_ctas=ctas, sk_maxseg=maxseg, sk_splits=splits,
                   sk_tiles=tiles, smem_bytes=smem + 64)
    return cfg


def stream_k_max_segments(tiles: int, kb: int, ctas: int) -> int:
    """The most CTAs whose stream-K ranges share one tile (the device's
    sk_lo / sk_owner arithmetic: CTA c owns iterations [c*I/G, (c+1)*I/G))."""
    total = tiles * kb

    def owner(x):
        c = x * ctas // total
        while c + 1 < ctas and (c + 1) * total // ctas <= x:
            c += 1
        while c > 0 and c * total // ctas > x:
            c -= 1
        return c
    return max(owner((t + 1) * kb - 1) - owner(t * kb) + 1 for t in range(tiles))


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
            "epi_warps": 4, "threads": 256, "smem_bytes": smem, "pair": True, "streamk": False}
