"""Parameter-Server RPC surface (C9).

The reference exposes admission/reserve/status to its Rust router over gRPC
(``psrl/grpc/ps_manager_service.py:33-216``).  Here the router runs in-process
or talks over :mod:`psrl_b200.utils.rpc`; this service keeps the same RPC
vocabulary so an external router can be wired to it unchanged in shape.
Errors are mapped to a ``(ok, error)`` envelope instead of raising across the
wire.
"""

from __future__ import annotations

from typing import Any

from .manager import PSManager
from .request_tracker import RequestStatus


def _envelope(fn):
    def wrapped(self, *a, **k) -> dict[str, Any]:
        try:
            return {"ok": True, "result": fn(self, *a, **k)}
        except Exception as exc:  # mapped error (the gRPC status in the reference)
            return {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
    wrapped.__name__ = fn.__name__
    return wrapped


class PSManagerService:
    def __init__(self, ps: PSManager):
        self.ps = ps

    @_envelope
    def CanReserveRequest(self, request_ids, model_versions, without_new_reserve_entry=False, is_validate=False):
        return self.ps.can_reserve_request(request_ids, list(model_versions), without_new_reserve_entry, is_validate)

    @_envelope
    def GetReserveIndicator(self, request_id, model_versions, is_validate=False):
        return self.ps.get_reserve_indicator(int(request_id), list(model_versions), is_validate)

    @_envelope
    def ReserveRolloutInstanceRequests(self, instance_ids, request_ids, model_versions, guarantee_not_aborted=True,
                                       is_validate=False):
        insts = [tuple(i) for i in instance_ids] if isinstance(instance_ids, list) else tuple(instance_ids)
        return self.ps.reserve_rollout_instance_requests(insts, request_ids, model_versions, guarantee_not_aborted,
                                                         is_validate)

    @_envelope
    def UpdateRequestInstanceId(self, request_id, instance_id, is_validate=False):
        return self.ps.update_request_instance_id(int(request_id), tuple(instance_id), is_validate)

    @_envelope
    def UpdateRequestVersionTag(self, request_id, version_tag, is_validate=False):
        return self.ps.update_request_version_tag(int(request_id), int(version_tag), is_validate)

    @_envelope
    def CheckAbortedRequests(self, request_ids, remove=False):
        return self.ps.check_aborted_requests(list(request_ids), remove)

    @_envelope
    def CheckAbortedModelVersions(self, model_versions):
        return self.ps.check_aborted_model_versions(list(model_versions))

    @_envelope
    def GetRolloutInstanceModelVersion(self, instance_id):
        return self.ps.get_rollout_instance_model_version(tuple(instance_id))

    @_envelope
    def UpdateRequestStatus(self, request_ids, status, model_version=-1, instance_id=(-1, -1), is_validate=False):
        st = RequestStatus[status] if isinstance(status, str) else status
        return self.ps.update_request_status(list(request_ids), st, model_version, tuple(instance_id), is_validate)

    @_envelope
    def GetPSModelVersion(self):
        return self.ps.get_ps_model_version()
