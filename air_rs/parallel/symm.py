"""Peer-memory (NVLink) fused collectives; filled in by the fused TP path."""


def maybe_fused_tp(tp, impl: str = "ours"):
    return tp
