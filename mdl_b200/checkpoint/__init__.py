"""Checkpoint storage, sharded reshardable model checkpoints, training checkpoints and resume."""

from .model import load_model_checkpoint, save_model_checkpoint
from .store import CheckpointStore, open_checkpoint_store
from .training import (DataCursor, latest_committed_checkpoint, list_committed_checkpoints,
                       load_training_checkpoint, make_uploader, prune_run_directory,
                       resolve_resume_checkpoint, save_training_checkpoint)
from .uploader import (CheckpointStagingSpaceError, CheckpointUploader, StagingEstimate, check_staging_space,
                       estimate_staging_bytes)

__all__ = [
    "CheckpointStagingSpaceError", "CheckpointUploader", "StagingEstimate", "check_staging_space",
    "estimate_staging_bytes", "make_uploader",
    "CheckpointStore", "DataCursor", "latest_committed_checkpoint", "list_committed_checkpoints",
    "load_model_checkpoint", "load_training_checkpoint", "open_checkpoint_store", "prune_run_directory",
    "resolve_resume_checkpoint", "save_model_checkpoint", "save_training_checkpoint",
]
