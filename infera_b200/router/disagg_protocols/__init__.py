"""Prefill/decode handoff protocols: how the two legs' bodies are shaped.

A protocol is stateless and shared; the router owns connections, retries
and metrics (interface of ``infera/router/disagg_protocols/base.py:20-91``).

* ``b200-nvlink-push`` (this framework's engines; concurrent): the prefill
  leg computes the prompt (one token) and pushes its KV pages straight into
  the decode instance's paged cache over NVLink; the decode leg parks until
  its room's pages arrived, recomputes only the last prompt token and
  generates the full token budget.
* body-shaping twins of the reference's protocols, kept so fleets that mix
  engines route identically: ``sglang-bootstrap`` (concurrent),
  ``vllm-mooncake`` (concurrent), ``vllm-mori-write`` (concurrent),
  ``vllm-mori-read`` and ``atom-mooncake`` (serial-pull).

:func:`resolve_protocol` requires the prefill and decode workers to
advertise the same ``disagg_meta["protocol"]``.
"""

from __future__ import annotations

from dataclasses import dataclass


def prefill_single_token(body: dict) -> dict:
    out = dict(body)
    out["max_tokens"] = 1
    out["stream"] = False
    out.pop("stream_options", None)
    if "max_completion_tokens" in out:
        out["max_completion_tokens"] = 1
    return out


def decode_remaining(body: dict) -> dict:
    out = dict(body)
    for k in ("max_tokens", "max_completion_tokens"):
        if isinstance(out.get(k), int):
            out[k] = max(1, out[k] - 1)
    return out


def _param(w, key: str, side: str):
    v = (w.disagg_meta.get("params") or {}).get(key)
    if v in (None, ""):
        raise ValueError(f"{side} worker {w.worker_id}: disagg_meta.params[{key!r}] missing")
    return v


@dataclass
class NvlinkPushProtocol:
    name: str = "b200-nvlink-push"
    topology: str = "concurrent"
    pin_prefill_dp_rank: bool = False

    def annotate_prefill(self, body, p, d, room_id):
        out = prefill_single_token(body)
        out["kv_transfer_params"] = {
            "do_remote_decode": True, "room": room_id, "decode_worker": d.worker_id,
            "decode_kv_endpoint": (d.disagg_meta.get("params") or {}).get("kv_endpoint"),
        }
        return out

    def annotate_decode(self, body, p, d, room_id, handoff):
        # the decode instance recomputes the last prompt token and samples
        # every output token itself: the full token budget stays with it
        out = dict(body)
        out["kv_transfer_params"] = {"do_remote_prefill": True, "room": room_id, "prefill_worker": p.worker_id}
        return out

    def extract_handoff(self, payload):
        return {}

    def request_id_for(self, p, d, room_id):
        return None


@dataclass
class SglangBootstrapProtocol:
    name: str = "sglang-bootstrap"
    topology: str = "concurrent"
    pin_prefill_dp_rank: bool = True

    def _fields(self, p, room_id):
        return {"bootstrap_host": _param(p, "bootstrap_host", "prefill"),
                "bootstrap_port": int(_param(p, "bootstrap_port", "prefill")), "bootstrap_room": room_id}

    def annotate_prefill(self, body, p, d, room_id):
        out = dict(body)
        out.update(self._fields(p, room_id))
        return out

    def annotate_decode(self, body, p, d, room_id, handoff):
        out = dict(body)
        out.update(self._fields(p, room_id))
        return out

    def extract_handoff(self, payload):
        return {}

    def request_id_for(self, p, d, room_id):
        return None


@dataclass
class VllmMooncakeProtocol:
    name: str = "vllm-mooncake"
    topology: str = "concurrent"
    pin_prefill_dp_rank: bool = True

    @staticmethod
    def transfer_id(room_id: int) -> str:
        return f"xfer-{room_id:032x}"

    def annotate_prefill(self, body, p, d, room_id):
        out = prefill_single_token(body)
        out["kv_transfer_params"] = {"do_remote_decode": True, "do_remote_prefill": False,
                                     "transfer_id": self.transfer_id(room_id)}
        return out

    def annotate_decode(self, body, p, d, room_id, handoff):
        out = decode_remaining(body)
        engine_id = _param(p, "engine_id", "prefill")
        if (p.dp_size or 1) > 1:
            engine_id = f"{engine_id}_dp{room_id % p.dp_size}"
        out["kv_transfer_params"] = {"do_remote_prefill": True, "do_remote_decode": False,
                                     "remote_engine_id": engine_id,
                                     "remote_bootstrap_addr": _param(p, "bootstrap_addr", "prefill"),
                                     "transfer_id": self.transfer_id(room_id)}
        return out

    def extract_handoff(self, payload):
        return {}

    def request_id_for(self, p, d, room_id):
        return None


@dataclass
class VllmMoriProtocol:
    """MoRI-IO: peer addressing travels in a forged request id."""

    name: str = "vllm-mori-read"
    topology: str = "serial-pull"
    pin_prefill_dp_rank: bool = False

    def request_id_for(self, p, d, room_id):
        ph = _param(p, "handshake_host", "prefill")
        pp = _param(p, "handshake_port", "prefill")
        dh = _param(d, "handshake_host", "decode")
        dp = _param(d, "handshake_port", "decode")
        return f"___prefill_addr_{ph}:{pp}___decode_addr_{dh}:{dp}_{room_id:x}"

    def annotate_prefill(self, body, p, d, room_id):
        out = prefill_single_token(body)
        out["kv_transfer_params"] = {"do_remote_decode": True, "do_remote_prefill": False}
        return out

    def annotate_decode(self, body, p, d, room_id, handoff):
        out = decode_remaining(body)
        ktp = {"do_remote_prefill": True, "do_remote_decode": False}
        ktp.update(handoff or {})
        out["kv_transfer_params"] = ktp
        return out

    def extract_handoff(self, payload):
        ktp = payload.get("kv_transfer_params") or {}
        return {k: ktp[k] for k in ("remote_block_ids", "remote_engine_id", "remote_host", "remote_port",
                                    "transfer_id") if k in ktp}


@dataclass
class VllmMoriWriteProtocol(VllmMoriProtocol):
    name: str = "vllm-mori-write"
    topology: str = "concurrent"


@dataclass
class AtomMooncakeProtocol(VllmMoriProtocol):
    name: str = "atom-mooncake"
    topology: str = "serial-pull"

    def request_id_for(self, p, d, room_id):
        return None


PROTOCOLS = {c().name: c() for c in (NvlinkPushProtocol, SglangBootstrapProtocol, VllmMooncakeProtocol,
                                     VllmMoriProtocol, VllmMoriWriteProtocol, AtomMooncakeProtocol)}


class ProtocolError(ValueError):
    pass


def protocol_of(w) -> str | None:
    return (w.disagg_meta or {}).get("protocol")


def resolve_protocol(p, d):
    pn, dn = protocol_of(p), protocol_of(d)
    if pn is None or dn is None:
        raise ProtocolError(f"worker without disagg protocol: prefill={pn!r} decode={dn!r}")
    if pn != dn:
        raise ProtocolError(f"protocol mismatch: prefill {p.worker_id}={pn!r} decode {d.worker_id}={dn!r}")
    proto = PROTOCOLS.get(pn)
    if proto is None:
        raise ProtocolError(f"unknown disagg protocol {pn!r}")
    return proto
