"""Drop-in for the reference's model-facing ``C4Adapter``
(sglang/srt/layers/attention/v1_deepseek/adapter.py:14-157): the opt-in C4
integration that turns a model batch into Indexer calls, one Indexer per local
compress-ratio-4 layer over that layer's native FP8 Index-K page-64 cache.

Behaviour kept from the reference (same names, argument meaning, checks and
error messages):
  * configuration (:24-71): SGLANG_V1_DEEPSEEK_CONFIG is a JSON object of Config
    fields plus the mandatory ``total_budget_bytes`` for all local layers; the
    head count defaults to the model's Index-Q heads.  Refused: outer CUDA
    graphs left on, tensor / pipeline parallelism, speculative decoding, either
    prefill context parallelism, the FP4 indexer, HiSparse, a topk or head count
    unlike the model's, a budget below the all-layer reservation, an index
    capacity below model context / 4, less free device memory than required;
  * row ownership (:73-102): a row belongs to ``(request slot, slot generation)``
    and sees ``len // 4`` compressed tokens -- a decode row its sequence length,
    the rows of an extend of ``count`` tokens after ``prefix`` the lengths
    ``prefix + 1 .. prefix + count``; padded batches are refused;
  * ``query`` (:104-143): the layer's native buffer is fetched from the
    backend's ``get_index_k_with_scale_buffer`` on every call and must keep its
    address; the page table is cut to ``Config.pages`` columns; results are
    copied into the caller's buffers (``raw_output`` receives the logical ids);
  * ``release_request(slot)`` drops every generation of a slot in every layer;
    ``clear()`` closes all layers so that a replacement native pool can bind.
"""
from __future__ import annotations

import json
import os

import torch

from .config import Config
from .indexer import Indexer

ENV = "SGLANG_V1_DEEPSEEK_CONFIG"


def _parse_config(raw: str, model_heads: int):
    fields = json.loads(raw)
    total = int(fields.pop("total_budget_bytes"))
    if "q_buckets" in fields:
        fields["q_buckets"] = tuple(fields["q_buckets"])
    fields.setdefault("heads", model_heads)
    return Config(**fields), total


def _unsupported_server(args, backend) -> bool:
    """Single-GPU FP8 without speculation, context parallelism or HiSparse only."""
    flags = (
        getattr(args, "tp_size", 1) != 1,
        getattr(args, "pp_size", 1) != 1,
        bool(getattr(args, "speculative_algorithm", None)),
        bool(getattr(args, "enable_prefill_context_parallel", False)),
        bool(getattr(args, "enable_dsa_prefill_context_parallel", False)),
        bool(backend.enable_deepseek_v4_fp4_indexer),
        backend.hisparse_coordinator is not None,
    )
    return any(flags)


def _local_c4_layers(backend) -> int:
    return sum(1 for item in backend.token_to_kv_pool.layer_mapping
               if item is not None and item.compress_ratio == 4)


class C4Adapter:
    def __init__(self, backend, config: Config, total_budget_bytes: int):
        self.backend = backend
        self.config = config
        self.total_budget_bytes = total_budget_bytes
        self.layers: dict[int, Indexer] = {}
        backend.req_to_token_pool.add_native_index_listener(self)

    @classmethod
    def from_environment(cls, backend):
        raw = os.environ.get(ENV)
        if not raw:
            return None
        heads = backend.model_runner.model_config.hf_text_config.index_n_heads
        config, total = _parse_config(raw, heads)
        if config.heads != heads:
            raise ValueError("V1 heads must match native Index Q heads")
        args = backend.model_runner.server_args
        if not (args.disable_cuda_graph and args.disable_prefill_cuda_graph):
            raise ValueError("V1 C4 subgraphs require --disable-cuda-graph --disable-prefill-cuda-graph; "
                             "inner graphs remain enabled")
        if _unsupported_server(args, backend):
            raise ValueError("V1 C4 currently supports single-GPU FP8 without speculation or HiSparse")
        if config.topk != backend.c4_topk:
            raise ValueError("V1 topk must match the native C4 attention topk")
        required = _local_c4_layers(backend) * config.reservation
        if total < required:
            raise ValueError(f"Total V1 budget {total} is below all-layer reservation {required}")
        if 4 * config.max_context < backend.max_context_len:
            raise ValueError("V1 index capacity must cover configured model context / 4")
        if required > torch.cuda.mem_get_info(backend.device)[0]:
            raise ValueError("Insufficient free GPU memory for V1; lower native mem-fraction-static")
        return cls(backend, config, total)

    # -- rows ----------------------------------------------------------------------
    def _owner(self, slot):
        return slot, int(self.backend.req_to_token_pool.req_generation[slot])

    def row_metadata(self, batch, rows):
        """(owners, compressed lengths) of the batch's query rows, in row order."""
        slots = batch.native_req_pool_indices_cpu
        if slots is None:
            raise ValueError("V1 C4 requires scheduler CPU request slots")
        mode = batch.forward_mode
        if mode.is_decode():
            if batch.seq_lens_cpu is None:
                raise ValueError("Missing scheduler CPU decode lengths")
            spans = [(slot, [int(n)]) for slot, n in zip(slots, batch.seq_lens_cpu.tolist())]
        elif mode.is_extend():
            prefixes, counts = batch.extend_prefix_lens_cpu, batch.extend_seq_lens_cpu
            if prefixes is None or counts is None:
                raise ValueError("Missing scheduler CPU prefill lengths")
            spans = [(slot, range(p + 1, p + c + 1)) for slot, p, c in zip(slots, prefixes, counts)]
        else:
            raise ValueError("V1 C4 does not support speculative/idle query dispatch")
        owners, lengths = [], []
        for slot, seen in spans:
            owner = self._owner(slot)
            for n in seen:
                owners.append(owner)
                lengths.append(max(0, n // 4))
        if len(owners) != rows:
            raise ValueError("V1 C4 requires unpadded scheduler-owned query rows")
        return owners, lengths

    # -- queries -------------------------------------------------------------------
    def _engine(self, layer, native):
        engine = self.layers.get(layer)
        if engine is None:
            if (len(self.layers) + 1) * self.config.reservation > self.total_budget_bytes:
                raise ValueError("All-layer V1 index reservation exceeds total_budget_bytes")
            engine = self.layers[layer] = Indexer(native, self.config)
        if native.data_ptr() != engine.native.data_ptr():
            raise RuntimeError("Native Index K buffer changed address; flush V1 before rebinding")
        return engine

    def query(self, c4_indexer, batch, q, weights, metadata, output, raw_output=None):
        if c4_indexer.use_fp4_indexer or metadata.c4_page_size != 64:
            raise ValueError("V1 C4 expects FP8 Index K with page_size=64")
        owners, lengths = self.row_metadata(batch, len(q))
        layer = c4_indexer.layer_id
        engine = self._engine(layer, self.backend.token_to_kv_pool.get_index_k_with_scale_buffer(layer_id=layer))
        table = metadata.page_table[:, :self.config.pages]
        result = engine.query(q.contiguous(), weights.float().contiguous(), table.contiguous(),
                              metadata.c4_seq_lens.reshape(-1).contiguous(), owners, lengths,
                              return_logical=raw_output is not None)
        if raw_output is None:
            output.copy_(result)
            return
        output.copy_(result[0])
        raw_output.copy_(result[1])

    def release_request(self, slot):
        for engine in self.layers.values():
            for owner in [o for o in engine.states if o[0] == slot]:
                engine.release_request(owner)

    def clear(self):
        for engine in self.layers.values():
            engine.close()
        self.layers.clear()
