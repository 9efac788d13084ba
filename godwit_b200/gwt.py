"""Loads a Godwit `.gwt` installation straight into the HBM-resident bank.

Format (restated from the reference, paths inside rayl15/Godwit):
  manifest.json  GodwitManifest (Install/GodwitManifest.swift:8-106): formatVersion
                 (2), spec (ArchitectureSpec: hiddenSize, intermediateSize,
                 activation, activationLimit, activationAlpha, routerBias,
                 layers[].expertsPerToken), layerCount, expertCount,
                 expertStride, expertSections {name: {offset, length}},
                 trunkSections [{name, offset, length, dtype, shape}].
  experts/layer_NN.bin
                 expertCount strides of expertStride bytes
                 (InstallLayout.swift:98-107, ModelReader.loadExpertStride :73-76).
  trunk.bin      router weights as trunk sections "layer{l}.router_w" (bf16
                 [E, H]) and "layer{l}.router_b" (bf16 [E], only when the spec
                 has a router bias) (Runtime/TransformerLayer.swift:55-60).

Each owned expert stride is read with one positional read into one of two
page-locked host buffers by a read-ahead thread while the other is uploaded
with gw_bank_upload_expert (a DMA copy from page-locked memory, then the
device re-layout), so the disk reads overlap the uploads.  A missing or inconsistent manifest is an
incomplete install and is rejected, as the reference does
(GodwitManifest.validate, ModelReader.swift:34-37).
"""
from __future__ import annotations

import json
import os
import queue
import threading

import numpy as np

from ._abi import GW_ACT_GPTOSS_CLAMPED, GW_ACT_SILU, GW_E_ARG, GW_E_UNSUPPORTED, SECTIONS, GodwitCUDAError
from .layout import ModelSpec

FORMAT_VERSION = 2
_ACTIVATIONS = {"gptOssClampedGLU": GW_ACT_GPTOSS_CLAMPED, "silu": GW_ACT_SILU}


class InstallError(GodwitCUDAError):
    def __init__(self, message: str):
        super().__init__(GW_E_ARG, message)


def read_manifest(root: str) -> dict:
    path = os.path.join(root, "manifest.json")
    if not os.path.exists(path):
        raise InstallError(f"{root} has no manifest.json: not a complete installation")
    m = json.load(open(path))
    if m.get("formatVersion") != FORMAT_VERSION:
        raise InstallError(f"manifest format {m.get('formatVersion')} is not {FORMAT_VERSION}")
    for s in SECTIONS:
        if s not in m.get("expertSections", {}):
            raise InstallError(f"manifest lacks expert section {s}")
    return m


def spec_of(m: dict) -> ModelSpec:
    s = m["spec"]
    act = s.get("activation")
    if act not in _ACTIVATIONS:
        raise GodwitCUDAError(GW_E_UNSUPPORTED, f"activation {act!r} has no kernel here")
    layers = s.get("layers") or [{}]
    return ModelSpec(
        name=m.get("model", "gwt"), hidden=int(s["hiddenSize"]),
        intermediate=int(s["intermediateSize"]), experts=int(m["expertCount"]),
        layers=int(m["layerCount"]), top_k=int(layers[0].get("expertsPerToken", 4)),
        activation=_ACTIVATIONS[act], limit=float(s.get("activationLimit", 7.0)),
        alpha=float(s.get("activationAlpha", 1.702)),
        expert_bias=bool(s.get("expertBias", True)), router_bias=bool(s.get("routerBias", True)))


def validate(root: str, m: dict) -> None:
    """Layer files present and exactly expertCount * expertStride bytes
    (GodwitManifest.validate, Install/GodwitManifest.swift:80-95)."""
    want = int(m["expertStride"]) * int(m["expertCount"])
    for layer in range(int(m["layerCount"])):
        p = layer_path(root, layer)
        if not os.path.exists(p):
            raise InstallError(f"layer {layer} file is unreadable")
        if os.path.getsize(p) != want:
            raise InstallError(f"layer {layer} is {os.path.getsize(p)} bytes, expected {want}")


def layer_path(root: str, layer: int) -> str:
    return os.path.join(root, "experts", f"layer_{layer:02d}.bin")


def _desc_from_manifest(bank_desc, m: dict) -> None:
    bank_desc.expert_stride = int(m["expertStride"])
    for i, s in enumerate(SECTIONS):
        span = m["expertSections"][s]
        bank_desc.section_offset[i] = int(span["offset"])
        bank_desc.section_length[i] = int(span["length"])


def load_bank(ctx, root: str, *, shard_rank: int = 0, shard_count: int = 1, layers=None):
    """Creates an ExpertBank holding the installation's experts (the owned
    shard) and routers.  Returns (bank, spec)."""
    from .runtime import ExpertBank
    m = read_manifest(root)
    validate(root, m)
    spec = spec_of(m)
    nl = spec.layers if layers is None else min(layers, spec.layers)

    # the descriptor takes the manifest's own stride and section spans
    desc = spec.desc(shard_rank, shard_count, nl)
    _desc_from_manifest(desc, m)
    bank = ExpertBank(ctx, spec, shard_rank=shard_rank, shard_count=shard_count, desc=desc)
    stride = int(m["expertStride"])
    bufs = staging_buffers(stride)
    trunk = _Trunk(root, m)
    for layer in range(nl):
        for e, buf in stream_strides(root, layer, range(shard_rank, spec.experts, shard_count), stride, bufs):
            bank.upload_expert(layer, e, buf)
        w = trunk.u16(f"layer{layer}.router_w", spec.experts * spec.hidden)
        b = trunk.u16(f"layer{layer}.router_b", spec.experts) if spec.router_bias else None
        bank.upload_router(layer, w, b)
    return bank, spec


def staging_buffers(stride: int, count: int = 2):
    """`count` host buffers of `stride` bytes, page-locked when a CUDA device
    is present (the uploads then DMA straight from them)."""
    try:
        import torch
        if torch.cuda.is_available():
            return [torch.empty(stride, dtype=torch.uint8, pin_memory=True).numpy() for _ in range(count)]
    except Exception:
        pass
    return [np.empty(stride, np.uint8) for _ in range(count)]


def stream_strides(root: str, layer: int, experts, stride: int, bufs):
    """Yields (expert, buffer) for each expert's stride of layer `layer`, read
    ahead by a thread into the buffers in turn (ModelReader.loadExpertStride,
    Runtime/ModelReader.swift:73-76).  A buffer is refilled only after the
    consumer has asked for the next stride, i.e. finished with it."""
    experts = list(experts)
    free: queue.Queue = queue.Queue()
    full: queue.Queue = queue.Queue()
    for i in range(len(bufs)):
        free.put(i)
    stop = threading.Event()

    def reader():
        # Every way out of this thread leaves the consumer something to take
        # from `full`: a stride, or the error that ended the reads.
        fd = None
        try:
            fd = os.open(layer_path(root, layer), os.O_RDONLY)
            for e in experts:
                i = free.get()
                if stop.is_set():
                    return
                n = os.preadv(fd, [memoryview(bufs[i])], e * stride)
                if n != stride:
                    full.put(InstallError(f"short read: layer {layer} expert {e} got {n} of {stride}"))
                    return
                full.put((e, i))
        except OSError as err:
            full.put(InstallError(f"layer {layer}: {err}"))
        except BaseException as err:  # noqa: BLE001 — reported to the consumer, not swallowed
            full.put(InstallError(f"layer {layer}: reader failed: {err!r}"))
        finally:
            if fd is not None:
                os.close(fd)

    t = threading.Thread(target=reader, daemon=True)
    t.start()
    try:
        for _ in experts:
            item = full.get()
            if isinstance(item, Exception):
                raise item
            e, i = item
            yield e, bufs[i]
            free.put(i)
    finally:
        stop.set()
        free.put(0)  # wakes a reader blocked on a buffer
        t.join()


class _Trunk:
    def __init__(self, root: str, m: dict):
        self.path = os.path.join(root, "trunk.bin")
        self.sections = {s["name"]: s for s in m.get("trunkSections", [])}

    def u16(self, name: str, count: int) -> np.ndarray:
        s = self.sections.get(name)
        if s is None:
            raise InstallError(f"trunk section {name} missing")
        if s.get("dtype", "bf16") != "bf16" or s["length"] != 2 * count:
            raise InstallError(f"trunk section {name} is not bf16 [{count}]")
        with open(self.path, "rb") as f:
            f.seek(s["offset"])
            raw = f.read(s["length"])
        if len(raw) != s["length"]:
            raise InstallError(f"trunk.bin is shorter than section {name}")
        return np.frombuffer(raw, dtype=np.uint16).copy()


def write_install(root: str, spec: ModelSpec, strides, routers, model: str = "synthetic") -> None:
    """Writes a minimal installation in the reference's format: manifest.json,
    experts/layer_NN.bin (strides [L][E][stride] uint8) and trunk.bin holding
    the router sections (routers [(w bf16 [E, H], b bf16 [E] or None)]).
    For tests and synthetic banks; the reference's installer writes the real
    ones from a checkpoint."""
    lay = spec.layout()
    os.makedirs(os.path.join(root, "experts"), exist_ok=True)
    for layer, st in enumerate(strides):
        np.ascontiguousarray(st, dtype=np.uint8).tofile(layer_path(root, layer))
    sections, cursor, page = [], 0, 16384
    with open(os.path.join(root, "trunk.bin"), "wb") as f:
        for layer, (w, b) in enumerate(routers):
            for name, arr in ((f"layer{layer}.router_w", w), (f"layer{layer}.router_b", b)):
                if arr is None:
                    continue
                cursor = (cursor + page - 1) // page * page
                raw = np.ascontiguousarray(arr, dtype=np.uint16).tobytes()
                f.seek(cursor)
                f.write(raw)
                sections.append({"name": name, "offset": cursor, "length": len(raw),
                                 "dtype": "bf16", "shape": list(np.shape(arr))})
                cursor += len(raw)
    act = {GW_ACT_GPTOSS_CLAMPED: "gptOssClampedGLU", GW_ACT_SILU: "silu"}[spec.activation]
    manifest = {
        "formatVersion": FORMAT_VERSION, "model": model, "revision": "synthetic",
        "spec": {"name": spec.name, "hiddenSize": spec.hidden,
                 "intermediateSize": spec.intermediate, "activation": act,
                 "activationLimit": spec.limit, "activationAlpha": spec.alpha,
                 "expertBias": spec.expert_bias, "routerBias": spec.router_bias,
                 "layers": [{"attention": "full", "window": 0,
                             "routedExpertCount": spec.experts,
                             "expertsPerToken": spec.top_k, "hasSharedExpert": False}
                            for _ in strides]},
        "layerCount": len(strides), "expertCount": spec.experts,
        "expertStride": lay.stride,
        "expertSections": {s: {"offset": lay.offsets[s], "length": lay.sizes[s]} for s in SECTIONS},
        "trunkSections": sections, "bytesWritten": 0,
    }
    with open(os.path.join(root, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
