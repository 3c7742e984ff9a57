"""B200 (sm_100a) RecoverSSM verify + grouped commit for Gated DeltaNet.

Drop-in replacement for the hot path of the ``gdn_recoverssm_ascend`` vLLM
plugin: the same entry points (``gdn_recoverssm_verify``,
``GDNRecoverSSMCommitContext``, ``GroupedCommitBucket``,
``GroupedCommitCoordinator``) backed by hand-written CUDA kernels exposed as
``torch.ops.gdn_recoverssm_ac.*`` over the C ABI in
``include/gdn_recoverssm_b200.h``.
"""

from .grouped_commit import CommitEntry, GroupedCommitBucket, GroupedCommitCoordinator
from .kernels import (
    MAX_SPEC_QUERY_LEN,
    NULL_BLOCK_ID,
    GDNRecoverSSMCommitContext,
    ReplayRecordBuffers,
    gdn_recoverssm_verify,
    gdn_recoverssm_verify_gated,
    record_geometry_bytes,
    record_nbytes,
)

__all__ = [
    "CommitEntry",
    "GDNRecoverSSMCommitContext",
    "GroupedCommitBucket",
    "GroupedCommitCoordinator",
    "MAX_SPEC_QUERY_LEN",
    "NULL_BLOCK_ID",
    "ReplayRecordBuffers",
    "gdn_recoverssm_verify",
    "gdn_recoverssm_verify_gated",
    "record_geometry_bytes",
    "record_nbytes",
]
