"""Python host of the B200 engine: owns one `sp_engine` (C ABI) per device.

PyTorch is used only for device memory and streams; all model arithmetic runs in the CUDA kernels
of `libseedplane_cuda.so`. Weights are accepted in two namings:

* HF names (`model.layers.{l}.self_attn.q_proj.weight`, ...), as a random-init checkpoint or a
  safetensors directory provides them, and
* seedplane-bundle/2 names (`embed`, `{l}.qkv_w`, `{l}.gate_w`, ...; `seedplane/native_bundle.py:106-120`).

Both are converted to the bundle-v2 layout the C ABI takes (fused QKV rows q|k|v, separate gate
and up, fp32 biases and norm gains).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence

import torch

from . import _native as N
from .config import Qwen2Config


def rope_table(cfg: Qwen2Config) -> torch.Tensor:
    """(cos, sin) [max_positions, head_dim/2, 2] fp32, computed like the reference on the CPU:
    fp32 inv_freq = 1/theta^(2i/HD), fp32 phase = pos * inv_freq (`qwen_engine.py:52,99-103`)."""
    hd = cfg.head_dim
    inv = 1.0 / (float(cfg.rope_theta) ** (torch.arange(0, hd, 2).float() / hd))
    phase = torch.outer(torch.arange(cfg.max_positions).float(), inv)
    return torch.stack([phase.cos(), phase.sin()], dim=-1).contiguous()


def hf_to_bundle_names(cfg: Qwen2Config, w: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """HF tensor names -> seedplane-bundle/2 names (QKV rows fused q|k|v, `native_bundle.py:112-114`)."""
    out = {"embed": w["model.embed_tokens.weight"], "final_norm": w["model.norm.weight"]}
    if "lm_head.weight" in w:
        out["lm_head"] = w["lm_head.weight"]
        if "lm_head.weight.scales" in w:
            out["lm_head.scales"] = w["lm_head.weight.scales"]
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        a = p + "self_attn."
        out[f"{l}.qkv_w"] = torch.cat([w[a + "q_proj.weight"], w[a + "k_proj.weight"], w[a + "v_proj.weight"]])
        out[f"{l}.qkv_b"] = torch.cat([w[a + "q_proj.bias"], w[a + "k_proj.bias"], w[a + "v_proj.bias"]])
        out[f"{l}.o_w"] = w[a + "o_proj.weight"]
        out[f"{l}.gate_w"] = w[p + "mlp.gate_proj.weight"]
        out[f"{l}.up_w"] = w[p + "mlp.up_proj.weight"]
        out[f"{l}.down_w"] = w[p + "mlp.down_proj.weight"]
        out[f"{l}.in_norm"] = w[p + "input_layernorm.weight"]
        out[f"{l}.post_norm"] = w[p + "post_attention_layernorm.weight"]
        if (a + "q_proj.weight.scales") in w:
            out[f"{l}.qkv_w.scales"] = torch.cat([w[a + "q_proj.weight.scales"], w[a + "k_proj.weight.scales"],
                                                  w[a + "v_proj.weight.scales"]])
            out[f"{l}.o_w.scales"] = w[a + "o_proj.weight.scales"]
            out[f"{l}.gate_w.scales"] = w[p + "mlp.gate_proj.weight.scales"]
            out[f"{l}.up_w.scales"] = w[p + "mlp.up_proj.weight.scales"]
            out[f"{l}.down_w.scales"] = w[p + "mlp.down_proj.weight.scales"]
    return out


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class DeviceKV:
    """One `sp_kv`: fp16 K/V of every layer, [layers][kv_heads][capacity][head_dim]."""

    def __init__(self, engine: "CudaQwen2", capacity: int):
        self.engine = engine
        h = C.c_void_p()
        N.check(N.load().sp_kv_create(engine.handle, int(capacity), C.byref(h)))
        self.handle = h

    @property
    def length(self) -> int:
        return int(N.load().sp_kv_length(self.handle))

    @length.setter
    def length(self, n: int):
        N.check(N.load().sp_kv_set_length(self.handle, int(n)))

    @property
    def capacity(self) -> int:
        return int(N.load().sp_kv_capacity(self.handle))

    def close(self):
        # sp_kv_destroy also frees a cache whose engine was destroyed first.
        if getattr(self, "handle", None) is not None:
            N.load().sp_kv_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaQwen2:
    """The CUDA engine for one Qwen2 checkpoint on one device."""

    def __init__(self, cfg: Qwen2Config, weights: Dict[str, torch.Tensor], device="cuda:0",
                 weight_format: str = "f16"):
        if not torch.cuda.is_available():
            raise RuntimeError("the SeedPlane B200 engine needs a CUDA device (there is no CPU fallback)")
        lib = N.load()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.int8 = weight_format == "i8"
        if "embed" not in weights:
            weights = hf_to_bundle_names(cfg, weights)
        dev = self.device
        keep: List[torch.Tensor] = []

        def mat(name):
            t = weights[name]
            if self.int8 and name != "embed":
                if t.dtype != torch.int8:
                    raise ValueError(f"{name}: int8 weights expected")
                t = t.to(dev).contiguous()
            else:
                t = t.to(device=dev, dtype=torch.float16).contiguous()
            keep.append(t)
            return t.data_ptr()

        def scales(name):
            if not self.int8:
                return None
            t = weights[name + ".scales"].to(device=dev, dtype=torch.float16).contiguous()
            keep.append(t)
            return t.data_ptr()

        def f32(name):
            t = weights[name].to(device=dev, dtype=torch.float32).contiguous()
            keep.append(t)
            return t.data_ptr()

        layers = (N.SpLayerWeights * cfg.layers)()
        for l in range(cfg.layers):
            L = layers[l]
            L.qkv_w, L.qkv_s, L.qkv_b = mat(f"{l}.qkv_w"), scales(f"{l}.qkv_w"), f32(f"{l}.qkv_b")
            L.o_w, L.o_s = mat(f"{l}.o_w"), scales(f"{l}.o_w")
            L.gate_w, L.gate_s = mat(f"{l}.gate_w"), scales(f"{l}.gate_w")
            L.up_w, L.up_s = mat(f"{l}.up_w"), scales(f"{l}.up_w")
            L.down_w, L.down_s = mat(f"{l}.down_w"), scales(f"{l}.down_w")
            L.in_norm, L.post_norm = f32(f"{l}.in_norm"), f32(f"{l}.post_norm")
        W = N.SpWeights()
        embed = weights["embed"].to(device=dev, dtype=torch.float16).contiguous()
        keep.append(embed)
        W.embed = embed.data_ptr()
        if not cfg.tied_embeddings:
            W.lm_head = mat("lm_head")
            W.lm_head_s = scales("lm_head")
        W.final_norm = f32("final_norm")
        W.layers = C.cast(layers, C.POINTER(N.SpLayerWeights))
        rope = rope_table(cfg)
        W.rope_host = rope.data_ptr()
        c = N.SpConfig(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads,
                       head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab,
                       max_positions=cfg.max_positions, rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps,
                       tied_embeddings=int(cfg.tied_embeddings),
                       weight_format=N.SP_WEIGHTS_I8_B32 if self.int8 else N.SP_WEIGHTS_F16)
        h = C.c_void_p()
        torch.cuda.synchronize(dev)
        N.check(lib.sp_engine_create(C.byref(c), C.byref(W), dev.index, C.byref(h)))
        self.handle = h
        del keep, rope
        torch.cuda.empty_cache()

    # ---------------------------------------------------------------------------------------
    def close(self):
        if getattr(self, "handle", None) is not None:
            N.load().sp_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return int(N.load().sp_engine_device_bytes(self.handle))

    def new_kv(self, capacity: int) -> DeviceKV:
        return DeviceKV(self, capacity)

    def status(self):
        """Raise if a kernel recorded a device-side error since the last check (syncs the stream)."""
        N.check(N.load().sp_device_status(self.handle, C.c_void_p(_stream(self.device))))

    def _ids(self, ids) -> torch.Tensor:
        t = torch.as_tensor(ids, dtype=torch.int32).flatten()
        return t.to(self.device, non_blocking=True)

    def forward(self, kv: DeviceKV, ids, positions=None, all_logits: bool = False, want_logits: bool = True,
                last_only: bool = False):
        """Qwen2Engine.forward semantics: logits fp32 [n or 1, V] (or None) and argmax int32 [n].
        `last_only`: the LM head for the last token alone (argmax int32 [1]); the others only fill
        the cache."""
        tok = ids if (isinstance(ids, torch.Tensor) and ids.device == self.device and ids.dtype == torch.int32) \
            else self._ids(ids)
        n = int(tok.numel())
        pos = None if positions is None else self._ids(positions)
        if pos is not None and pos.numel() != n:
            raise ValueError("positions must match input_ids")
        if last_only and all_logits:
            raise ValueError("last_only excludes all_logits")
        logits = None
        if want_logits:
            logits = torch.empty((n if all_logits else 1, self.cfg.vocab), dtype=torch.float32, device=self.device)
        argmax = torch.empty(1 if last_only else n, dtype=torch.int32, device=self.device)
        N.check(N.load().sp_forward(self.handle, kv.handle, C.c_void_p(tok.data_ptr()),
                                    C.c_void_p(pos.data_ptr() if pos is not None else None), n,
                                    C.c_void_p(logits.data_ptr() if logits is not None else None),
                                    2 if last_only else int(all_logits), C.c_void_p(argmax.data_ptr()),
                                    C.c_void_p(_stream(self.device))))
        return logits, argmax

    def decode(self, kv: DeviceKV, token: int, pos: int, n_steps: int, out: Optional[torch.Tensor] = None,
               want_logits: bool = False):
        """Greedy device-fed decode of n_steps tokens; returns (tokens int32 [n_steps], last logits or None)."""
        if out is None:
            out = torch.empty(n_steps, dtype=torch.int32, device=self.device)
        logits = torch.empty(self.cfg.vocab, dtype=torch.float32, device=self.device) if want_logits else None
        N.check(N.load().sp_decode(self.handle, kv.handle, int(token), int(pos), int(n_steps),
                                   C.c_void_p(out.data_ptr()),
                                   C.c_void_p(logits.data_ptr() if logits is not None else None),
                                   C.c_void_p(_stream(self.device))))
        return out, logits

    def decode_batch(self, kvs: Sequence[DeviceKV], tokens: Sequence[int], positions: Sequence[int], n_steps: int,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Greedy decode of len(kvs) independent requests together (`sp_decode_batch`): request b feeds
        tokens[b] at positions[b] into kvs[b]; returns the argmaxes int32 [n_steps, B]."""
        B = len(kvs)
        if out is None:
            out = torch.empty((n_steps, B), dtype=torch.int32, device=self.device)
        handles = (C.c_void_p * B)(*[kv.handle for kv in kvs])
        N.check(N.load().sp_decode_batch(self.handle, handles, B, N.int_array(tokens), N.int_array(positions),
                                         int(n_steps), C.c_void_p(out.data_ptr()), C.c_void_p(_stream(self.device))))
        return out

    def prefill_batch(self, kvs: Sequence[DeviceKV], prompts: Sequence[Sequence[int]]) -> torch.Tensor:
        """The prompts of len(kvs) requests in packed batched passes (`sp_prefill_batch`): prompt b is
        appended to kvs[b]; returns the greedy token after each prompt, int32 [B]."""
        B = len(kvs)
        flat = torch.tensor([int(t) for p in prompts for t in p], dtype=torch.int32).to(self.device, non_blocking=True)
        out = torch.empty(B, dtype=torch.int32, device=self.device)
        handles = (C.c_void_p * B)(*[kv.handle for kv in kvs])
        N.check(N.load().sp_prefill_batch(self.handle, handles, B, C.c_void_p(flat.data_ptr()),
                                          N.int_array([len(p) for p in prompts]), C.c_void_p(out.data_ptr()),
                                          C.c_void_p(_stream(self.device))))
        return out

    def verify_tree(self, kv: DeviceKV, tokens: Sequence[int], parents: Sequence[int], base_pos: int,
                    want_logits: bool = False):
        """One batched pass over a draft tree; returns (argmax int32 [n], logits [n, V] or None)."""
        n = len(tokens)
        argmax = torch.empty(n, dtype=torch.int32, device=self.device)
        logits = torch.empty((n, self.cfg.vocab), dtype=torch.float32, device=self.device) if want_logits else None
        N.check(N.load().sp_verify_tree(self.handle, kv.handle, N.int_array(tokens), N.int_array(parents), n,
                                        int(base_pos), C.c_void_p(logits.data_ptr() if logits is not None else None),
                                        C.c_void_p(argmax.data_ptr()), C.c_void_p(_stream(self.device))))
        return argmax, logits

    def kv_commit(self, kv: DeviceKV, src_slots: Sequence[int]):
        N.check(N.load().sp_kv_commit(kv.handle, N.int_array(src_slots), len(src_slots),
                                      C.c_void_p(_stream(self.device))))

    def kv_copy(self, src: DeviceKV, src_slot0: int, dst: DeviceKV, dst_slot0: int, n: int):
        """K/V of slots [src_slot0, src_slot0 + n) of `src` into [dst_slot0, ...) of `dst` (every
        layer; lengths unchanged): `sp_kv_copy`."""
        N.check(N.load().sp_kv_copy(src.handle, int(src_slot0), dst.handle, int(dst_slot0), int(n),
                                    C.c_void_p(_stream(self.device))))

    def topk(self, logits: torch.Tensor, k: int):
        """Per-row top-k of fp32 logits on the device: (indices int32 [rows, k], values [rows, k],
        log-sum-exp [rows]); larger value first, lower index on ties."""
        x = logits if logits.dim() == 2 else logits.reshape(1, -1)
        if x.dtype != torch.float32 or x.device != self.device or x.stride(1) != 1:
            raise ValueError("topk wants fp32 logits on the engine's device, rows contiguous")
        rows, cols = x.shape
        idx = torch.empty((rows, k), dtype=torch.int32, device=self.device)
        val = torch.empty((rows, k), dtype=torch.float32, device=self.device)
        lse = torch.empty(rows, dtype=torch.float32, device=self.device)
        N.check(N.load().sp_topk(self.handle, C.c_void_p(x.data_ptr()), rows, cols, x.stride(0), k,
                                 C.c_void_p(idx.data_ptr()), C.c_void_p(val.data_ptr()), C.c_void_p(lse.data_ptr()),
                                 C.c_void_p(_stream(self.device))))
        return idx, val, lse

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        """Row-wise greedy argmax (lowest index on ties) of fp32 logits [rows, V] on this device."""
        if logits.device != self.device or logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("fp32 logits [rows, V] with unit column stride on the engine's device expected")
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=self.device)
        N.check(N.load().sp_argmax(self.handle, C.c_void_p(logits.data_ptr()), logits.shape[0], logits.shape[1],
                                   logits.stride(0), C.c_void_p(out.data_ptr()), C.c_void_p(_stream(self.device))))
        return out


    def mcol_gemm(self, w: torch.Tensor, x: torch.Tensor, *, mode: str = "store", w_lo: Optional[torch.Tensor] = None,
                  alpha: float = 1.0, y: Optional[torch.Tensor] = None, act: Optional[tuple] = None) -> torch.Tensor:
        """The batched pass's projection (`sp_mcol_gemm`): alpha * W . x^T on the tcgen05 multi-column
        GEMM, x split into fp16 hi / lo halves here. w: fp16 [N, K] (w_lo: a second half, W = w + w_lo);
        x: fp32 [T, K]. mode "store" returns y [T, N]; "resid" adds into the given y [T, N]; "swiglu"
        (rows 2i gate, 2i + 1 up) writes SiLU(gate) * up as fp16 hi / lo into act = (hi, lo) [T, N / 2]
        and returns their sum as fp32."""
        T, K = x.shape
        Nrows = w.shape[0]
        xs = torch.zeros((2 * T, K), dtype=torch.float16, device=self.device)
        xf = x.to(self.device, torch.float32)
        xs[:T] = xf.half()
        xs[T:] = (xf - xs[:T].float()).half()
        modes = {"store": 0, "resid": 1, "swiglu": 2}
        if mode == "store":
            y = torch.empty((T, Nrows), dtype=torch.float32, device=self.device)
        elif mode == "swiglu":
            act = act or (torch.empty((T, Nrows // 2), dtype=torch.float16, device=self.device),
                          torch.empty((T, Nrows // 2), dtype=torch.float16, device=self.device))
        ptr = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
        N.check(N.load().sp_mcol_gemm(self.handle, modes[mode], ptr(w), ptr(w_lo), float(alpha), Nrows, K, ptr(xs),
                                      2 * T, T, T, ptr(y), Nrows, ptr(act[0]) if act else None,
                                      ptr(act[1]) if act else None, Nrows // 2, C.c_void_p(_stream(self.device))))
        if mode == "swiglu":
            return act[0].float() + act[1].float()
        return y

def argmax_noalloc(logits: torch.Tensor) -> torch.Tensor:
    """Row-wise greedy argmax of fp32 logits [rows <= 128, V] through `sp_argmax_noalloc`: no engine
    and no device allocation in the library (its scratch is a fixed device array). Calls on one
    device must not overlap in time; the first call on a device must precede any stream capture."""
    if logits.device.type != "cuda" or logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("fp32 CUDA logits [rows, V] with unit column stride expected")
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    N.check(N.load().sp_argmax_noalloc(logits.device.index, C.c_void_p(logits.data_ptr()), logits.shape[0],
                                       logits.shape[1], logits.stride(0), C.c_void_p(out.data_ptr()),
                                       C.c_void_p(_stream(logits.device))))
    return out
