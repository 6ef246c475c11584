"""``LRKV_LATENT``: the attention backend over the latent KV cache of ``latent`` exports, with the decode path on this
package's sm_100a kernels. Mirrors the reference's ``vllm_lrkv.latent_backend``
(plugins/vllm_lrkv/vllm_lrkv/latent_backend.py): same classes, constructor arguments, ``forward`` /
``do_kv_cache_update`` signatures, metadata fields and error behaviour.

Every compressed layer keeps one BF16 row per token in its own page (``LatentKVSpec``: one head slot of ``row_width``
elements, no separate V). The model hands the op the normed, rotated query ([T, H, head_dim]), the latent projection
of every new token as the "key" and the positions as the "value". The op first writes the tokens' cache rows
(``latent_ops.latent_rows_to_cache``; on a second stream when the step has ``SIDE_STREAM_MIN_DECODES`` decodes or
more, joined before the decode reads the cache), then:

* decode (one query token per request, at the front of the batch): the block-diagonal query, the split-KV decode
  kernel over the paged rows on the step's schedule (computed once per step by the builder and shared by all layers),
  the merge of each request's segments and the per-head V up-projection written straight into ``output``;
* prefill (everything else): for all prefill requests of the step together, keys and values rebuilt from the rows
  gathered through the block table in one tcgen05 launch (``LatentLayer.decompress_varlen``) and causal attention on
  the tensor cores in one more (``latent_ops.prefill_attention_varlen``), in rounds of at most ``PREFILL_CHUNK``
  context tokens whose results are folded by log-sum-exp (``latent_ops.attn_fold``).

When the running vLLM provides the plugin API the reference targets (``vllm_plugin.vllm_api``), the backend, the KV
spec and the attention-type / block-size types are vLLM's own classes (``LatentAttentionBackend`` subclasses vLLM's
``AttentionBackend``, ``LatentKVSpec`` its ``FullAttentionSpec``); without it, stand-ins of the same shape are used and
the package runs on its own. ``vllm_plugin.register`` installs the backend into vLLM.
"""

from __future__ import annotations

from dataclasses import dataclass
import os
from typing import ClassVar

import torch

from . import decode as dec
from . import latent_ops, vllm_plugin
from .layer import LatentLayer

BACKEND_NAME = "LRKV_LATENT"
PREFILL_CHUNK = int(os.environ.get("LRKV_PREFILL_CHUNK_TOKENS", 32768))
SIDE_STREAM_MIN_DECODES = int(os.environ.get("LRKV_SIDE_STREAM_MIN_DECODES", 32))


class _StandInAttentionType:
    DECODER = "decoder"
    ENCODER = "encoder"
    ENCODER_ONLY = "encoder_only"
    ENCODER_DECODER = "encoder_decoder"


@dataclass(frozen=True)
class _StandInMultipleOf:
    base: int


def make_kv_spec_class(api):
    """``LatentKVSpec``: one compressed layer's cache, a single head slot of ``head_size`` (the row width) elements per
    token and no separate V (latent_backend.py:57-62), on vLLM's ``FullAttentionSpec`` when ``api`` provides it."""
    if api is not None:
        @dataclass(frozen=True, kw_only=True)
        class LatentKVSpec(api.FullAttentionSpec):
            """One compressed layer's cache: one head slot of the row width per token, no separate V."""

            head_size_v: int = 0
        return LatentKVSpec

    @dataclass(frozen=True, kw_only=True)
    class LatentKVSpec:
        """One compressed layer's cache: one head slot of the row width per token, no separate V."""

        block_size: int
        num_kv_heads: int = 1
        head_size: int = 0
        dtype: torch.dtype = torch.bfloat16
        head_size_v: int = 0

        @property
        def page_size_bytes(self) -> int:
            return self.block_size * self.num_kv_heads * self.head_size * torch.finfo(self.dtype).bits // 8
    return LatentKVSpec


_API = vllm_plugin.vllm_api()
AttentionType = _API.AttentionType if _API is not None else _StandInAttentionType
MultipleOf = _API.MultipleOf if _API is not None else _StandInMultipleOf
LatentKVSpec = make_kv_spec_class(_API)


@dataclass
class CommonAttentionMetadata:
    """The per-step batch description the builder consumes (the fields of vLLM's ``CommonAttentionMetadata`` that the
    reference's builder reads)."""

    query_start_loc: torch.Tensor           # [num_reqs + 1] int32, device
    query_start_loc_cpu: torch.Tensor       # [num_reqs + 1] int32, host
    seq_lens: torch.Tensor                  # [num_reqs] int32, device (this step's tokens included)
    block_table_tensor: torch.Tensor        # [num_reqs, max_blocks] int32
    slot_mapping: torch.Tensor              # [num_actual_tokens] int64 / int32
    num_reqs: int
    num_actual_tokens: int
    max_query_len: int = 1
    seq_lens_cpu_upper_bound: torch.Tensor | None = None


def split_decodes_and_prefills(cm: CommonAttentionMetadata, decode_threshold: int = 1):
    """(num_decodes, num_prefills, num_decode_tokens, num_prefill_tokens) of a batch reordered with its decode requests
    (query length <= decode_threshold) first (vLLM's ``split_decodes_and_prefills``)."""
    qsl = cm.query_start_loc_cpu
    n = cm.num_reqs
    if cm.max_query_len <= decode_threshold:
        return n, 0, cm.num_actual_tokens, 0
    q_len = (qsl[1:n + 1] - qsl[:n]).tolist()
    nd = 0
    while nd < n and q_len[nd] <= decode_threshold:
        nd += 1
    ndt = int(qsl[nd])
    return nd, n - nd, ndt, cm.num_actual_tokens - ndt


@dataclass
class LatentAttentionMetadata:
    num_actual_tokens: int
    num_decodes: int
    num_decode_tokens: int
    num_prefills: int
    num_prefill_tokens: int
    block_table: torch.Tensor           # [num_reqs, max_blocks] int32
    seq_lens: torch.Tensor              # [num_reqs] int32, including this step's tokens
    sched: dec.DecodeSchedule | None    # the decode requests' work split, filled for this step
    slot_mapping: torch.Tensor | None = None
    prefill_cu_q: torch.Tensor | None = None
    prefill_cu_k: torch.Tensor | None = None
    prefill_max_q: int = 0
    prefill_max_k: int = 0
    prefill_q_len: list | None = None
    prefill_seq_len: list | None = None


_LAST_BUILD: dict = {}
_SCHEDULES: dict = {}
_SIDE_STREAMS: dict = {}
_ERROR_WATCHES: dict = {}


class _ErrorWatch:
    """Reads a device's error word (``decode.error_word``) one step late, without a synchronisation: every build
    enqueues a copy of the word into pinned host memory behind the work already queued, and the next build reads that
    copy if it has landed (otherwise the check waits for a later build). A nonzero word means a bounded wait inside a
    kernel gave up on an earlier step, so that step's output is not valid: the build raises ``BeltError`` (and clears
    the word). Nothing is enqueued or read while the stream is capturing a CUDA graph."""

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.landed = torch.cuda.Event()
        self.armed = False

    def poll(self) -> None:
        if torch.cuda.is_current_stream_capturing():
            return
        _warn_on_fallbacks()
        if self.armed:
            if not self.landed.query():
                return                              # the GPU is still behind: read at a later build
            self.armed = False
            code = int(self.host[0])
            if code:
                dec.error_word(self.device).zero_()
                from ._lib import BeltError
                raise BeltError(f"device error 0x{code:x} recorded by a belt kernel on {self.device} in an earlier "
                                "step: its attention output is not valid")
        stream = torch.cuda.current_stream(self.device)
        self.host.copy_(dec.error_word(self.device), non_blocking=True)
        self.landed.record(stream)
        self.armed = True


_FALLBACKS_SEEN: dict = {}


def _warn_on_fallbacks() -> None:
    """Warn once per kind when a launch took a CUDA-core fallback (operands TMA cannot describe: a strided query or
    latent view with rows not 16-byte aligned, a group over more than five 64-column chunks). The results are correct;
    the fallback is slower."""
    import warnings
    from . import _lib
    for kind, n in _lib.path_counts().items():
        if n > _FALLBACKS_SEEN.get(kind, 0):
            if kind not in _FALLBACKS_SEEN:
                warnings.warn(f"belt_b200: {n} launch(es) took the CUDA-core fallback ({kind}): the operands' strides or "
                              "alignment cannot be described by TMA", RuntimeWarning, stacklevel=3)
            _FALLBACKS_SEEN[kind] = n


def _error_watch(device: torch.device) -> _ErrorWatch:
    w = _ERROR_WATCHES.get(device)
    if w is None:
        w = _ERROR_WATCHES[device] = _ErrorWatch(device)
    return w


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    """The device's second stream for the cache rows (created at the first such step, before any graph capture)."""
    stream = _SIDE_STREAMS.get(device)
    if stream is None:
        stream = _SIDE_STREAMS[device] = torch.cuda.Stream(device)
    return stream


def _write_rows(m: LatentAttentionMetadata, device, write):
    """Run ``write`` (this step's cache rows): on the side stream when the step has ``SIDE_STREAM_MIN_DECODES`` decodes
    or more (it then overlaps the absorbed query; the caller joins the returned stream before reading the cache), else
    on the current stream (returns None)."""
    if m.num_decodes >= SIDE_STREAM_MIN_DECODES:
        main, side = torch.cuda.current_stream(device), _side_stream(device)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            write()
        return side
    write()
    return None


class LatentAttentionMetadataBuilder:
    """Per-step metadata; fills the step's decode schedule once (latent_backend.py:148-225)."""

    reorder_batch_threshold: int = 1
    cudagraph_support: ClassVar[str] = "UNIFORM_SINGLE_TOKEN_DECODE"

    def __init__(self, kv_cache_spec: LatentKVSpec, layer_names, vllm_config=None, device=None,
                 max_num_batched_tokens: int = 8192):
        self.kv_cache_spec = kv_cache_spec
        self.layer_names = layer_names
        self.device = torch.device(device if device is not None else "cuda")
        self.block_size = kv_cache_spec.block_size
        if vllm_config is not None:
            max_num_batched_tokens = vllm_config.scheduler_config.max_num_batched_tokens
        if self.device not in _SCHEDULES:
            _SCHEDULES[self.device] = dec.make_schedule(max_num_batched_tokens, self.device)
        self.sched = _SCHEDULES[self.device]

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> LatentAttentionMetadata:
        cm = common_attn_metadata
        last = _LAST_BUILD.get(self.device)
        if last is not None and last[0] is cm and last[1] == self.block_size:
            return last[2]
        m = self._build(cm)
        _LAST_BUILD[self.device] = (cm, self.block_size, m)
        return m

    def _build(self, cm: CommonAttentionMetadata) -> LatentAttentionMetadata:
        _error_watch(self.device).poll()
        nd, npf, ndt, npt = split_decodes_and_prefills(cm, decode_threshold=1)
        m = LatentAttentionMetadata(num_actual_tokens=cm.num_actual_tokens, num_decodes=nd, num_decode_tokens=ndt,
                                    num_prefills=npf, num_prefill_tokens=npt, block_table=cm.block_table_tensor,
                                    seq_lens=cm.seq_lens, sched=self.sched if nd else None,
                                    slot_mapping=cm.slot_mapping)
        if nd:
            dec.schedule(self.sched, cm.seq_lens[:nd])
        if npf:
            qsl = cm.query_start_loc_cpu[nd:nd + npf + 1].to(torch.int64)
            if cm.seq_lens_cpu_upper_bound is not None:
                seq_cpu = cm.seq_lens_cpu_upper_bound[nd:nd + npf].to(torch.int64)
            else:
                seq_cpu = cm.seq_lens[nd:nd + npf].to("cpu", torch.int64)
            m.prefill_q_len = (qsl[1:] - qsl[:-1]).tolist()
            m.prefill_seq_len = seq_cpu.tolist()
            m.prefill_max_q = max(m.prefill_q_len)
            m.prefill_max_k = max(m.prefill_seq_len)
        return m


class LatentAttentionImpl:
    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes: list | None = None, sliding_window: int | None = None, kv_cache_dtype: str = "auto",
                 logits_soft_cap: float | None = None, attn_type: str = AttentionType.DECODER,
                 kv_sharing_target_layer_name: str | None = None, **kwargs) -> None:
        if (attn_type != AttentionType.DECODER or alibi_slopes is not None or sliding_window is not None
                or logits_soft_cap or kv_sharing_target_layer_name is not None):
            raise NotImplementedError("LRKV_LATENT: causal decoder self-attention only (no alibi, sliding window, "
                                      "soft cap or KV sharing)")
        if kv_cache_dtype not in ("auto", "bfloat16"):
            raise NotImplementedError(f"LRKV_LATENT keeps a BF16 latent cache, not {kv_cache_dtype}")
        self.num_heads, self.head_size, self.scale = num_heads, head_size, scale
        self.num_kv_heads = num_kv_heads or num_heads
        self.kv_cache_dtype = kv_cache_dtype

    def do_kv_cache_update(self, layer, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
        """key: the latent projection [T, pe_offset] of the new tokens, value: their positions (unused)."""
        lat: LatentLayer = layer.latent
        latent_ops.latent_rows_to_cache(key, slot_mapping, kv_cache[:, 0], lat.u_cat, lat.k_segs_host, lat.eps)

    def forward(self, layer, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                attn_metadata: LatentAttentionMetadata, output: torch.Tensor, output_scale=None,
                output_block_scale=None) -> torch.Tensor:
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("LRKV_LATENT: fused output quantization")
        if attn_metadata is None:                 # profiling run
            return output.fill_(0)
        m = attn_metadata
        slots = m.slot_mapping
        side = None
        if slots is not None and key is not None:
            side = _write_rows(m, query.device, lambda: self.do_kv_cache_update(layer, key, value, kv_cache, slots))
        return self._attend(layer, query, kv_cache, m, output, side)

    def _attend(self, layer, query: torch.Tensor, kv_cache: torch.Tensor, m: LatentAttentionMetadata,
                output: torch.Tensor, side) -> torch.Tensor:
        """Decode and prefill attention of the step; ``side`` is the stream still writing this step's rows (or None):
        the decode waits for it after the absorbed query, which does not read the cache."""
        lat: LatentLayer = layer.latent
        cache = kv_cache[:, 0]                    # [blocks, block_size, row_width], strided per block
        nd = m.num_decode_tokens
        if m.num_decodes:
            dev = query.device
            q_bd = lat.block_diag_query(query[:nd])
            if side is not None:
                torch.cuda.current_stream(dev).wait_stream(side)   # the step's own rows are part of the context
                side = None
            part = dec.partial_buffer(nd + m.sched.num_ctas, lat.v_rank, dev)
            lse = torch.empty(nd, self.num_heads, dtype=torch.float32, device=dev)
            dec.latent_decode(q_bd, cache, m.block_table[:nd], m.seq_lens[:nd], m.sched, part, self.scale,
                              lat.v_offset, lat.v_rank, rope=lat.rope)
            # the segment merge and the U_v projection in one kernel, straight into the output rows
            dec.merge_up_project(part, m.sched, lat.v_up, output[:nd], lse)
        if side is not None:
            torch.cuda.current_stream(query.device).wait_stream(side)
        if m.num_prefills:
            self._prefill(lat, query, output, cache, m)
        return output

    def _prefill(self, lat: LatentLayer, query: torch.Tensor, output: torch.Tensor, cache: torch.Tensor,
                 m: LatentAttentionMetadata) -> None:
        """Every prefill request's new tokens over its whole context, causal (latent_backend.py:285-320), all requests
        of the step together: per round of at most ``PREFILL_CHUNK`` context tokens (``plan_prefill_rounds``), one
        launch rebuilds the round's keys and values from the cache rows on the tensor cores
        (``latent_ops.decompress_varlen``) and one runs the attention of every request over its part of them
        (``latent_ops.prefill_attention_varlen``); the first part of a request writes its output rows directly, later
        parts are folded into them by log-sum-exp (``latent_ops.attn_fold``, the reference's ``merge_attn_states``)."""
        nd, tok0 = m.num_decodes, m.num_decode_tokens
        qls, lens = m.prefill_q_len, m.prefill_seq_len
        npt = sum(qls)
        q_rel = [sum(qls[:i]) for i in range(len(qls))]       # rows of each request's tokens from tok0 on
        q, out = query[tok0:tok0 + npt], output[tok0:tok0 + npt]
        dev = query.device
        lse = torch.empty(npt, self.num_heads, dtype=torch.float32, device=dev)
        tmp = tmp_lse = None
        for rnd in plan_prefill_rounds(lens, PREFILL_CHUNK):
            k, v = lat.decompress_varlen(cache, m.block_table, [(nd + i, lens[i], k0, k1 - k0) for i, k0, k1 in rnd])
            att, fold, krow = [], [], 0
            for i, k0, k1 in rnd:
                later = k0 > 0
                att.append((q_rel[i], qls[i], krow, k1 - k0, lens[i] - qls[i], k0, q_rel[i], int(later)))
                if later:
                    fold.append((q_rel[i], q_rel[i], qls[i]))
                krow += k1 - k0
            if fold and tmp is None:
                tmp = torch.empty_like(out)
                tmp_lse = torch.empty_like(lse)
            latent_ops.prefill_attention_varlen(q, k, v, att, self.scale, out, lse, tmp, tmp_lse, causal=True)
            if fold:
                latent_ops.attn_fold(out, lse, tmp, tmp_lse, fold)


def plan_prefill_rounds(seq_lens, chunk: int) -> list:
    """The key ranges a prefill step rebuilds, round by round: [(request index, k0, k1), ...] per round, at most
    ``chunk`` keys in all per round (``chunk`` <= 0: one round of whole contexts). Every request's ranges cover
    [0, seq_len) in order, the first starting at 0, at most one range of a request per round."""
    if chunk <= 0:
        return [[(i, 0, int(L)) for i, L in enumerate(seq_lens) if L > 0]]
    rounds, cur, used = [], [], 0
    for i, L in enumerate(seq_lens):
        k = 0
        while k < L:
            take = min(int(L) - k, chunk - used)
            cur.append((i, k, k + take))
            used += take
            k += take
            if used == chunk:
                rounds.append(cur)
                cur, used = [], 0
    if cur:
        rounds.append(cur)
    return rounds


def latent_attention_step(impl: "LatentAttentionImpl", layer, query: torch.Tensor, hidden: torch.Tensor,
                          w_down: torch.Tensor, kv_cache: torch.Tensor, attn_metadata: LatentAttentionMetadata,
                          output: torch.Tensor) -> torch.Tensor:
    """The attention half of one compressed layer as the model runs it (models/qwen3_5_latent.py:204-217:
    ``key = kv_latent_proj(hidden)``, then the backend's cache write and attention), with the down-projection fused
    into the cache write: the rows of every scheduled token (``attn_metadata.slot_mapping``) are computed from
    ``hidden`` [T, hidden_size] and ``w_down`` (``kv_latent_proj.weight`` [>= row_width, hidden_size]) and written in
    one kernel (on the side stream at ``SIDE_STREAM_MIN_DECODES`` decodes, overlapping the absorbed query, as
    ``LatentAttentionImpl.forward`` does with its cache write), then attends as ``impl.forward``."""
    if attn_metadata is None:
        return output.fill_(0)
    lat: LatentLayer = layer.latent
    m = attn_metadata
    side = None
    if m.slot_mapping is not None:
        side = _write_rows(m, query.device, lambda: latent_ops.project_rows_to_cache(
            hidden, w_down, m.slot_mapping, kv_cache[:, 0], lat.u_cat, lat.k_segs_host, lat.eps))
    return impl._attend(layer, query, kv_cache, m, output, side)


def make_backend_class(api):
    """``LatentAttentionBackend`` (latent_backend.py:322-354) on vLLM's ``AttentionBackend`` when ``api`` provides it,
    its block-size and layout types taken from the same API."""
    base = api.AttentionBackend if api is not None else object
    multiple_of = api.MultipleOf if api is not None else _StandInMultipleOf
    layouts = (api.KVCacheLayout.BLHNC, api.KVCacheLayout.BLNHC) if api is not None else ("BLHNC", "BLNHC")

    class LatentAttentionBackend(base):
        # This backend writes the cache rows itself (inside forward); vLLM is told not to call a separate update, which
        # also keeps the slot mapping padded to the key's token count, the layout the row-writing kernel reads.
        forward_includes_kv_cache_update: bool = False
        accept_output_buffer: bool = True
        supported_dtypes: ClassVar[list] = [torch.bfloat16]
        supported_kv_cache_dtypes: ClassVar[list] = ["auto", "bfloat16"]

        @staticmethod
        def get_name() -> str:
            return BACKEND_NAME

        @staticmethod
        def get_impl_cls() -> type[LatentAttentionImpl]:
            return LatentAttentionImpl

        @staticmethod
        def get_builder_cls() -> type[LatentAttentionMetadataBuilder]:
            return LatentAttentionMetadataBuilder

        @staticmethod
        def get_supported_kernel_block_sizes(kv_cache_spec=None) -> list:
            # the decode kernel's tile is 128 tokens fetched as boxes of one page: 16, 32, 64 or a multiple of 128
            return [16, 32, 64, multiple_of(128)]

        @classmethod
        def supports_head_size(cls, head_size: int) -> bool:
            return True

        @classmethod
        def supported_kv_cache_layouts(cls):
            """Block-major layouts only. Every compressed layer has its own row width, so the pages of one block sit
            next to each other per layer, which needs the block index outermost."""
            return layouts

    return LatentAttentionBackend


LatentAttentionBackend = make_backend_class(_API)


def register_with_vllm() -> bool:
    """Register the backend under ``LRKV_LATENT`` (and the KV-cache hooks) in a vLLM that provides the plugin API the
    reference targets; returns False when it does not (``vllm_plugin.register``)."""
    return vllm_plugin.register()
