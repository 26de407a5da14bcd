from ssd.models.bridges import RMSNorm, TransitionBridge
from ssd.models.subnetwork_draft import BridgeSpec, DraftOutput, SubnetworkDraftModel

__all__ = ["RMSNorm", "TransitionBridge", "BridgeSpec", "DraftOutput", "SubnetworkDraftModel"]
