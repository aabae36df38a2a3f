"""suika_b200: a B200-native drop-in for the data path of Suika's live state migration.

Public entry points mirror Suika/migration.py: schedule_param_transfer, execute_param_transfer,
schedule_and_execute_param_transfer (the drop-in used by migration_save / migration_load), plus
reshard_local (all ranks of a reshard emulated on one device). Around them:
  suika_b200.handoff     old -> new process hand-off (Suika/utils.py:325-406)
  suika_b200.metadata    layouts exchanged as planner records (Suika/migration.py:172-192)
  suika_b200.activation  activation hand-over between pipeline stages (Suika/pipeline_parallel.py:665-836)
"""
from .migration import (ParamLayout, Plan, Program, TensorMeta, TransferOp, get_param_tensor_meta,  # noqa: F401
                        is_ib_enabled, launch_copies)

__version__ = "0.1.0"
