"""CudaModel: batched decode of a Llama-architecture model on B200 through libpox_cuda.so.

Host-side mirror of the reference's decode interface: PoxEngine::forward_token(token, pos,
&mut KvCache) -> logits (crates/paraoxidizer-runtime/src/engine.rs:411-716) and the greedy
sampler (crates/paraoxidizer-runtime/src/sampler.rs:55-65), for a batch of sequences whose KV
cache lives in fp16 pages of 16 tokens tracked by the BlockManager / BlockTable bookkeeping of
paged_cache.rs (paged.py). Weights are the .pox payloads the reference's `pox quantize` writes:
INT4 g128 projections (optional outlier tables), f16 embedding / lm_head / norms.
"""
from __future__ import annotations

import ctypes as C
import weakref
from typing import Optional, Sequence

import numpy as np

from . import _lib as L
from .paged import DEFAULT_BLOCK_SIZE, BlockManager, BlockTable

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a)).view(np.uint8).reshape(-1)


def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint16)).reshape(-1)


class CudaModel:
    """A model resident on one B200: weights uploaded once, paged fp16 KV cache in HBM.

    With tp_size > 1 this object is rank tp_rank of a tensor-parallel model (one process per GPU):
    it takes the rank's weight shards (tp.shard_llama), returns the rank's vocab slice of the
    logits, and needs init_comm() on every rank before the first step."""

    def __init__(self, backend, cfg: dict, max_batch: int, kv_blocks: int, max_blocks_per_seq: int,
                 tp_rank: int = 0, tp_size: int = 1):
        self.backend = backend
        self.cfg = dict(cfg)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        c = L.LlamaConfig(cfg["hidden"], cfg["inter"], cfg["layers"], cfg["n_heads"], cfg["n_kv_heads"],
                          cfg["vocab"], np.float32(cfg.get("rms_eps", 1e-5)), np.float32(cfg.get("rope_theta", 500000.0)))
        h = C.c_void_p()
        L.check(L.lib().pox_cuda_model_create_tp(backend.ctx, C.byref(c), max_batch, kv_blocks, max_blocks_per_seq,
                                                 tp_rank, tp_size, C.byref(h)))
        self.handle = h.value
        backend._children.append(weakref.ref(self))
        self.max_batch = max_batch
        self.max_blocks_per_seq = max_blocks_per_seq
        self.blocks = BlockManager(kv_blocks, DEFAULT_BLOCK_SIZE)

    @classmethod
    def from_pox(cls, backend, pox_file, max_batch: int, kv_blocks: int, max_blocks_per_seq: int, tp_rank: int = 0,
                 tp_size: int = 1) -> "CudaModel":
        """The model of a .pox file (pox_format.PoxFile), rank tp_rank of tp_size, uploaded once
        (pox_cuda_model_load); its configuration is the file's model_config."""
        cfg = pox_file.model_config()
        h = C.c_void_p()
        L.check(L.lib().pox_cuda_model_load(backend.ctx, pox_file.handle, max_batch, kv_blocks, max_blocks_per_seq,
                                            tp_rank, tp_size, C.byref(h)))
        self = cls.__new__(cls)
        self.backend = backend
        self.cfg = {k: v for k, v in cfg.items() if k != "tie_word_embeddings"}
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.handle = h.value
        backend._children.append(weakref.ref(self))
        self.max_batch = max_batch
        self.max_blocks_per_seq = max_blocks_per_seq
        self.blocks = BlockManager(kv_blocks, DEFAULT_BLOCK_SIZE)
        return self

    @property
    def vocab_local(self) -> int:
        return self.cfg["vocab"] // self.tp_size

    def init_comm(self, modes=("peer", "nccl"), group=None) -> None:
        """Sets up the tensor-parallel exchanges (collective over the torch.distributed group of
        the tp_size ranks, rank order = tp_rank): "nccl" joins an NCCL communicator, "peer" maps
        every rank's exchange buffer over CUDA IPC. The first mode listed is selected."""
        import torch.distributed as dist

        lib = L.lib()
        for mode in modes:
            if mode == "nccl":
                uid = (C.c_uint8 * 128)()
                if self.tp_rank == 0:
                    L.check(lib.pox_cuda_comm_unique_id(uid))
                obj = [bytes(uid)]
                dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0, group=group)
                buf = (C.c_uint8 * 128).from_buffer_copy(obj[0])
                L.check(lib.pox_cuda_model_comm_nccl(self.handle, buf))
            elif mode == "peer":
                h = (C.c_uint8 * 64)()
                L.check(lib.pox_cuda_model_comm_ipc_handle(self.handle, h))
                hs = [None] * self.tp_size
                dist.all_gather_object(hs, bytes(h), group=group)
                allh = (C.c_uint8 * (64 * self.tp_size)).from_buffer_copy(b"".join(hs))
                L.check(lib.pox_cuda_model_comm_peer(self.handle, allh))
            else:
                raise ValueError(f"unknown exchange {mode!r}")
        self.set_comm_mode(modes[0])
        dist.barrier(group=group)  # every rank's buffers exist and are mapped before the first step

    def set_comm_mode(self, mode: str) -> None:
        L.check(L.lib().pox_cuda_model_comm_mode(self.handle, {"nccl": L.POX_COMM_NCCL, "peer": L.POX_COMM_PEER}[mode]))

    def set_persistent(self, enable: bool) -> None:
        """True: decode steps of batch 1-4 run every layer as one persistent kernel when the model
        qualifies (pox_cuda_model_set_persistent); False (the default) keeps one launch per projection."""
        L.check(L.lib().pox_cuda_model_set_persistent(self.handle, 1 if enable else 0))

    def step_persistent(self, batch: int) -> bool:
        """Whether a decode step of `batch` rows runs as the persistent kernel."""
        return bool(L.lib().pox_cuda_model_step_persistent(self.handle, batch))

    def close(self) -> None:
        if self.handle:
            L.lib().pox_cuda_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ------------------------------------------------------------------------
    def set_embeddings(self, embed, final_norm, lm_head) -> None:
        e, f, hd = _u16(embed), _u16(final_norm), _u16(lm_head)
        L.check(L.lib().pox_cuda_model_set_embeddings(self.handle, e.ctypes.data, f.ctypes.data, hd.ctypes.data))

    def set_layer(self, layer: int, proj: dict, attn_norm, mlp_norm) -> None:
        """proj[name] = {"packed", "scales", "rows", "cols", "group_size", "outliers": .pox table bytes or None}
        for name in q, k, v, o, gate, up, down."""
        descs = (L.TensorDesc * 7)()
        keep = []
        for i, name in enumerate(PROJ):
            t = proj[name]
            p, s = _u8(t["packed"]), _u8(t["scales"])
            o = None if t.get("outliers") is None else _u8(t["outliers"])
            keep += [p, s, o]
            d = descs[i]
            d.dtype, d.rows, d.cols, d.group_size = L.POX_I4, t["rows"], t["cols"], t["group_size"]
            d.data, d.data_len = p.ctypes.data, p.size
            d.scales, d.scale_len = s.ctypes.data, s.size
            d.outliers, d.outlier_len = (None, 0) if o is None else (o.ctypes.data, o.size)
        a, m = _u16(attn_norm), _u16(mlp_norm)
        L.check(L.lib().pox_cuda_model_set_layer(self.handle, layer, descs, a.ctypes.data, m.ctypes.data))

    def set_embeddings_device(self, embed_ptr: int, final_norm_ptr: int, lm_head_ptr: int) -> None:
        """Same as set_embeddings with device pointers (f16 [vocab][hidden], [hidden], [vocab][hidden])."""
        L.check(L.lib().pox_cuda_model_set_embeddings(self.handle, embed_ptr, final_norm_ptr, lm_head_ptr))

    def set_layer_tensors(self, layer: int, qkv: int, o: int, gate_up: int, down: int, attn_norm, mlp_norm) -> None:
        """Adopts resident tensors (handles of pox_tensor) as layer `layer`; see
        pox_cuda_model_set_layer_tensors."""
        a, m = _u16(attn_norm), _u16(mlp_norm)
        L.check(L.lib().pox_cuda_model_set_layer_tensors(self.handle, layer, qkv, o, gate_up, down, a.ctypes.data,
                                                         m.ctypes.data))

    # ---- decode -------------------------------------------------------------------------
    def new_sequence(self) -> BlockTable:
        return BlockTable(DEFAULT_BLOCK_SIZE)

    def decode(self, tokens: Sequence[int], seqs: Sequence[BlockTable], want_logits: bool = True):
        """One forward_token per sequence (engine.rs:411-716) at its next position; appends the
        token to each sequence's block table. Returns (logits [batch][vocab / tp_size] (this rank's
        vocab slice) or None, greedy next tokens [batch])."""
        B = len(tokens)
        assert B == len(seqs) and B > 0
        pos = np.zeros(B, np.uint32)
        tab = np.full((B, self.max_blocks_per_seq), -1, np.int32)
        for b, s in enumerate(seqs):
            pos[b] = s.sequence_len
            s.append_token(self.blocks)
            tab[b] = s.as_array(self.max_blocks_per_seq)
        tok = np.asarray(tokens, np.uint32)
        logits = np.zeros((B, self.vocab_local), np.float32) if want_logits else None
        nxt = np.zeros(B, np.uint32)
        L.check(L.lib().pox_cuda_model_decode(self.handle, B, tok.ctypes.data, pos.ctypes.data, tab.ctypes.data,
                                              None if logits is None else logits.ctypes.data, nxt.ctypes.data))
        return logits, nxt

    def prefill(self, prompts: Sequence[Sequence[int]], seqs: Sequence[BlockTable], want_logits: bool = True):
        """Feeds each sequence's prompt tokens at its next positions in passes of up to max_batch rows
        (pox_cuda_model_prefill; the tensor-core GEMMs see all rows of a pass at once). Returns the
        logits of each sequence's last prompt token ([n_seq][vocab / tp_size], or None) and the greedy
        next tokens, like forward_token on the last prompt token (engine.rs:758-762)."""
        assert len(prompts) == len(seqs) and len(seqs) > 0
        rows = []  # (sequence, token, position)
        for i, (p, s) in enumerate(zip(prompts, seqs)):
            for tok in p:
                rows.append((i, int(tok), s.sequence_len))
                s.append_token(self.blocks)
        last = {}
        for r, (i, _, _) in enumerate(rows):
            last[i] = r
        n = len(seqs)
        logits = np.zeros((n, self.vocab_local), np.float32) if want_logits else None
        nxt = np.zeros(n, np.uint32)
        lib = L.lib()
        for c0 in range(0, len(rows), self.max_batch):
            chunk = rows[c0:c0 + self.max_batch]
            tok = np.array([t for _, t, _ in chunk], np.uint32)
            pos = np.array([p for _, _, p in chunk], np.uint32)
            tab = np.stack([seqs[i].as_array(self.max_blocks_per_seq) for i, _, _ in chunk]).astype(np.int32)
            outs = [(i, r - c0) for i, r in last.items() if c0 <= r < c0 + len(chunk)]
            sel = np.array([r for _, r in outs] or [len(chunk) - 1], np.uint32)
            lg = np.zeros((len(sel), self.vocab_local), np.float32)
            nx = np.zeros(len(sel), np.uint32)
            L.check(lib.pox_cuda_model_prefill(self.handle, len(chunk), tok.ctypes.data, pos.ctypes.data,
                                               tab.ctypes.data, len(sel), sel.ctypes.data,
                                               lg.ctypes.data if want_logits else None, nx.ctypes.data))
            for j, (i, _) in enumerate(outs):
                nxt[i] = nx[j]
                if want_logits:
                    logits[i] = lg[j]
        return logits, nxt

    def set_state(self, tokens, seqs: Sequence[BlockTable]) -> None:
        """Loads tokens, the sequences' next positions and their block tables into the device
        buffers (pox_cuda_model_set_state) for decode_device steps."""
        B = len(tokens)
        pos = np.array([s.sequence_len for s in seqs], np.uint32)
        tab = np.stack([s.as_array(self.max_blocks_per_seq) for s in seqs]).astype(np.int32)
        tok = np.asarray(tokens, np.uint32)
        L.check(L.lib().pox_cuda_model_set_state(self.handle, B, tok.ctypes.data, pos.ctypes.data, tab.ctypes.data))

    def buffers(self):
        ptrs = [C.c_void_p() for _ in range(5)]
        L.check(L.lib().pox_cuda_model_buffers(self.handle, *[C.byref(p) for p in ptrs]))
        return [p.value for p in ptrs]  # tokens, positions, block tables, logits, next

    def decode_device(self, batch: int, advance: bool, stream: int = 0) -> None:
        """Asynchronous step on the model's device buffers (see pox_cuda_model_decode_device)."""
        L.check(L.lib().pox_cuda_model_decode_device(self.handle, batch, None, None, None, None, None,
                                                     1 if advance else 0, stream or None))
