"""Torch-facing wrappers over the C ABI: tensors in, raw pointers to the library.

Every op runs on the caller's current CUDA stream, checks dtypes, devices and
contiguity on the host, and raises ``ValueError`` (bad arguments, as the
reference does) or ``RuntimeError`` (CUDA failure). Outputs are written into
caller-provided tensors; nothing here allocates device memory except where an
op's docstring says it returns a new tensor.
"""

from __future__ import annotations

import torch

from helios_b200 import _native

BF16 = torch.bfloat16
TICK_ROW_FIELDS = 7  # slot, length, count, logit count, pages, shared prefix keys, group rows
DECODE_ITEM_INTS = 6  # row, first key, end key, record base, splits of the row, 0
PREFIX_ITEM_INTS = 5  # first row, rows, first key, end key, prefix split index


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, *, contiguous: bool = True) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def lib():
    return _native.load()


def tick_pack(rows_dev: torch.Tensor, num_rows: int, updates_dev: torch.Tensor | None, num_updates: int,
              arena: torch.Tensor, page_size: int, width: int, num_pages: int, decode_max_tokens: int,
              split_keys: int, prefill_tile_tokens: int, total_tokens: int, out: dict, *,
              prefix_split_keys: int | None = None) -> None:
    """Kernel (a): expand row descriptors into the tick's metadata (``out`` holds the buffers)."""
    _need(rows_dev, torch.int32, "rows")
    _need(arena, torch.int32, "arena")
    rc = lib().hb_tick_pack(
        rows_dev.data_ptr(), num_rows, _ptr(updates_dev) if num_updates else None, num_updates, arena.data_ptr(),
        arena.shape[0], arena.shape[1], page_size, width, num_pages, decode_max_tokens, split_keys,
        prefill_tile_tokens, split_keys if prefix_split_keys is None else prefix_split_keys, total_tokens,
        out["block_table"].data_ptr(), out["cu_seq_q"].data_ptr(), out["cu_seq_k"].data_ptr(),
        out["seqused_k"].data_ptr(), out["positions"].data_ptr(), out["write_slots"].data_ptr(),
        out["token_row"].data_ptr(), out["logit_store"].data_ptr(), out["logit_store"].numel(),
        out["decode_items"].data_ptr(), out["decode_items"].numel() // DECODE_ITEM_INTS,
        out["prefill_items"].data_ptr(), out["prefill_items"].numel() // 3,
        _ptr(out.get("prefix_items")), out["prefix_items"].numel() // PREFIX_ITEM_INTS if "prefix_items" in out else 0,
        _ptr(out.get("counts")),
        _ptr(out.get("row_records")), _stream(rows_dev.device))
    _native.check(rc, "hb_tick_pack")


def qk_norm_rope_append(q: torch.Tensor | None, k: torch.Tensor, v: torch.Tensor, *, q_scale, k_scale, eps: float,
                        cos, sin, positions, write_slots: torch.Tensor, q_out: torch.Tensor | None,
                        key_pool: torch.Tensor, value_pool: torch.Tensor) -> None:
    """Kernel (b). q/k/v are ``[T, heads, d]`` views (any token/head strides, unit
    element stride); pools are one layer ``[P, page, Hkv, d]``."""
    tokens, kv_heads, dim = k.shape
    heads = q.shape[1] if q is not None else kv_heads
    for name, t in (("k", k), ("v", v)) + ((("q", q),) if q is not None else ()):
        _need(t, BF16, name, contiguous=False)
        if t.stride(-1) != 1:
            raise ValueError(f"{name} rows must be contiguous along head_dim")
    _need(key_pool, BF16, "key_pool")
    _need(value_pool, BF16, "value_pool")
    if q_out is not None:
        _need(q_out, BF16, "q_out")
    if write_slots.dtype != torch.long:
        raise ValueError("write_slots must be int64")
    pool_slots = key_pool.shape[0] * key_pool.shape[1]
    rc = lib().hb_qk_norm_rope_append(
        _ptr(q), q.stride(0) if q is not None else 0, q.stride(1) if q is not None else 0,
        k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1),
        _ptr(q_scale), _ptr(k_scale), float(eps), _ptr(cos), _ptr(sin), cos.shape[0] if cos is not None else 0,
        _ptr(positions), write_slots.data_ptr(), _ptr(q_out), key_pool.data_ptr(), value_pool.data_ptr(),
        pool_slots, tokens, heads, kv_heads, dim, _stream(k.device))
    _native.check(rc, "hb_qk_norm_rope_append")


def workspace_bytes(partial_records: int, heads: int, head_dim: int) -> int:
    return int(lib().hb_attention_workspace_bytes(partial_records, heads, head_dim))


def paged_attention(q: torch.Tensor, key_pool: torch.Tensor, value_pool: torch.Tensor, meta, out: torch.Tensor,
                    *, scale: float | None = None) -> torch.Tensor:
    """Kernel (c): ``q [T, H, d]`` against the paged pool described by ``meta``
    (a prepared paged batch cache); writes ``out [T, H, d]``. A cache in capacity mode
    passes its device work counts and launches grids sized to its capacities."""
    _need(q, BF16, "q")
    _need(out, BF16, "out")
    _need(key_pool, BF16, "key_pool")
    _need(value_pool, BF16, "value_pool")
    tokens, heads, dim = q.shape
    kv_heads = key_pool.shape[2]
    scale = dim ** -0.5 if scale is None else scale
    ws = meta.workspace
    rc = lib().hb_paged_attention(
        q.data_ptr(), key_pool.data_ptr(), value_pool.data_ptr(), key_pool.shape[0], key_pool.shape[1],
        meta.block_table.data_ptr(), meta.block_table.shape[1], meta.cu_seq_q.data_ptr(), meta.seqused_k.data_ptr(),
        meta.batch_size, meta.row_records.data_ptr(),
        meta.decode_items.data_ptr(), meta.launch_decode_items, meta.prefill_items.data_ptr(),
        meta.launch_prefill_items, meta.prefix_items.data_ptr(), meta.launch_prefix_items,
        _ptr(meta.attention_counts), meta.launch_partial_records, meta.split_keys, tokens,
        heads, kv_heads, dim, float(scale),
        _ptr(ws), ws.numel() if ws is not None else 0, out.data_ptr(), _stream(q.device))
    _native.check(rc, "hb_paged_attention")
    return out


def rmsnorm(x: torch.Tensor, scale: torch.Tensor, eps: float, *, out: torch.Tensor | None = None,
            row_index: torch.Tensor | None = None) -> torch.Tensor:
    """Row RMSNorm of ``x [rows, hidden]`` (rows gathered by ``row_index`` first)."""
    _need(x, BF16, "x")
    _need(scale, torch.float32, "scale")
    rows = x.shape[0] if row_index is None else row_index.shape[0]
    if out is None:
        out = torch.empty(rows, x.shape[1], dtype=BF16, device=x.device)
    if row_index is not None and row_index.dtype != torch.long:
        raise ValueError("row_index must be int64")
    rc = lib().hb_rmsnorm(x.data_ptr(), x.shape[0], _ptr(row_index), scale.data_ptr(), float(eps), out.data_ptr(),
                          rows, x.shape[1], _stream(x.device))
    _native.check(rc, "hb_rmsnorm")
    return out


def add_rmsnorm(x: torch.Tensor, y: torch.Tensor, scale: torch.Tensor, eps: float, sum_out: torch.Tensor,
                norm_out: torch.Tensor) -> None:
    """``sum_out = bf16(x + y)``; ``norm_out = rmsnorm(sum_out)``."""
    for name, t in (("x", x), ("y", y), ("sum_out", sum_out), ("norm_out", norm_out)):
        _need(t, BF16, name)
    _need(scale, torch.float32, "scale")
    rc = lib().hb_add_rmsnorm(x.data_ptr(), y.data_ptr(), scale.data_ptr(), float(eps), sum_out.data_ptr(),
                              norm_out.data_ptr(), x.shape[0], x.shape[1], _stream(x.device))
    _native.check(rc, "hb_add_rmsnorm")


def swiglu(gate_up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    _need(gate_up, BF16, "gate_up")
    _need(out, BF16, "out")
    if gate_up.shape[1] != 2 * out.shape[1] or gate_up.shape[0] != out.shape[0]:
        raise ValueError("gate_up must be [rows, 2 * inter] for out [rows, inter]")
    rc = lib().hb_swiglu(gate_up.data_ptr(), out.data_ptr(), gate_up.shape[0], out.shape[1], _stream(out.device))
    _native.check(rc, "hb_swiglu")
    return out


def gemm_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(x Wg^T) * (x Wu^T)`` with the reference's bf16 rounding points, for ``x [m, k]``
    and the fused ``w_gate_up [2 * inter, k]`` (gate rows then up rows), on tcgen05."""
    _need(x, BF16, "x")
    _need(w_gate_up, BF16, "w_gate_up")
    m, k = x.shape
    inter = w_gate_up.shape[0] // 2
    if w_gate_up.shape[1] != k or w_gate_up.shape[0] != 2 * inter:
        raise ValueError("w_gate_up must be [2 * intermediate, hidden] matching x")
    if out is None:
        out = torch.empty((m, inter), dtype=BF16, device=x.device)
    rc = lib().hb_gemm_swiglu(x.data_ptr(), m, k, w_gate_up.data_ptr(), inter, out.data_ptr(), _stream(x.device))
    _native.check(rc, "hb_gemm_swiglu")
    return out


# Buffers a larger call replaced: kept alive, since a CUDA graph captured earlier still
# launches kernels on their addresses.
_RETIRED: list[torch.Tensor] = []


_ARGMAX_KEYS: dict[torch.device, torch.Tensor] = {}


def lm_head_argmax(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token ids ``argmax_j bf16(x[r] . weight[j])`` (int64 ``[m]``; ties to the lowest id)
    for the final-normed logit rows ``x [m, k]`` against the tied ``weight [vocab, k]``, with the
    argmax in the tcgen05 GEMM's epilogue: the logits are never written (hb_lm_head_argmax)."""
    _need(x, BF16, "x")
    _need(weight, BF16, "weight")
    m, k = x.shape
    if weight.shape[1] != k:
        raise ValueError("weight must be [vocab, hidden] matching x")
    dev = x.device
    keys = _ARGMAX_KEYS.get(dev)
    if keys is None or keys.numel() < m:
        if torch.cuda.is_current_stream_capturing():
            # Memory allocated under capture belongs to the graph's pool; the keys outlive graphs.
            raise RuntimeError("lm_head_argmax: run one call of this size before capturing it")
        # Zeroed once; every call leaves the keys it used at zero.
        if keys is not None:
            _RETIRED.append(keys)
        keys = _ARGMAX_KEYS[dev] = torch.zeros(max(m, 256), dtype=torch.int64, device=dev)
    if out is None:
        out = torch.empty(m, dtype=torch.long, device=dev)
    rc = lib().hb_lm_head_argmax(x.data_ptr(), m, k, weight.data_ptr(), weight.shape[0], keys.data_ptr(),
                                 out.data_ptr(), _stream(dev))
    _native.check(rc, "hb_lm_head_argmax")
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    if ids.dtype != torch.long or not ids.is_cuda or not ids.is_contiguous():
        raise ValueError("token ids must be a contiguous CUDA int64 tensor")
    _need(table, BF16, "table")
    _need(out, BF16, "out")
    rc = lib().hb_embedding(ids.data_ptr(), table.data_ptr(), table.shape[0], out.data_ptr(), ids.numel(),
                            table.shape[1], _stream(out.device))
    _native.check(rc, "hb_embedding")
    return out


def page_copy(storage: torch.Tensor, src_pages: torch.Tensor, dst_pages: torch.Tensor) -> None:
    """Copy pages ``src -> dst`` in every pool tensor of ``storage [tensors, P, ...]``."""
    if src_pages.dtype != torch.int32 or dst_pages.dtype != torch.int32:
        raise ValueError("page lists must be int32")
    tensors, num_pages = storage.shape[0], storage.shape[1]
    page_bytes = storage[0, 0].numel() * storage.element_size()
    rc = lib().hb_page_copy(storage.data_ptr(), storage.stride(0) * storage.element_size(), tensors, page_bytes,
                            num_pages, src_pages.data_ptr(), dst_pages.data_ptr(), src_pages.numel(),
                            _stream(storage.device))
    _native.check(rc, "hb_page_copy")


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_p: torch.Tensor, uniforms: torch.Tensor,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Kernel (d): one token id per row of bf16 ``logits [rows, V]`` (row stride may exceed V)."""
    _need(logits, BF16, "logits", contiguous=False)
    if logits.stride(1) != 1:
        raise ValueError("logit rows must be contiguous")
    for name, t in (("temperature", temperature), ("top_p", top_p), ("uniforms", uniforms)):
        _need(t, torch.float32, name)
    rows, vocab = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.long, device=logits.device)
    rc = lib().hb_sample(logits.data_ptr(), logits.stride(0), rows, vocab, temperature.data_ptr(), top_p.data_ptr(),
                         uniforms.data_ptr(), out.data_ptr(), _stream(logits.device))
    _native.check(rc, "hb_sample")
    return out


def verify_drafts(tokens: torch.Tensor, cu_seq_q: torch.Tensor, logit_offsets: torch.Tensor,
                  predictions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Speculative verification on the device: ``(accepted [B] int32, emitted [logit rows]
    int64)``; row r's emitted tokens are ``emitted[logit_offsets[r] : logit_offsets[r] +
    accepted[r] + 1]`` (engine.py:507-520)."""
    _need(tokens, torch.long, "tokens")
    _need(cu_seq_q, torch.int32, "cu_seq_q")
    _need(logit_offsets, torch.int32, "logit_offsets")
    _need(predictions, torch.long, "predictions")
    rows = cu_seq_q.numel() - 1
    if logit_offsets.numel() != rows + 1:
        raise ValueError("logit_offsets needs one entry per row plus one")
    accepted = torch.empty(rows, dtype=torch.int32, device=tokens.device)
    emitted = torch.zeros(predictions.numel(), dtype=torch.long, device=tokens.device)
    rc = lib().hb_verify_drafts(tokens.data_ptr(), cu_seq_q.data_ptr(), logit_offsets.data_ptr(),
                                predictions.data_ptr(), rows, accepted.data_ptr(), emitted.data_ptr(),
                                _stream(tokens.device))
    _native.check(rc, "hb_verify_drafts")
    return accepted, emitted
