"""Model-agnostic runtime: training engine, checkpoints, loggers, metrics."""

from .callbacks import EarlyStopping, LearningRateMonitor, ModelCheckpoint, ProgressPrinter
from .checkpointing import CheckpointError, atomic_save, load_checkpoint, read_checkpoint, serializable_config
from .logging import ConsoleLogger, ExperimentLogger, MultiLogger, TensorBoardLogger, build_logger
from .metrics import DeviceTimer, RunningAverages, ThroughputTimer, cuda_memory_allocated, grad_norm, perplexity
from .plots import MetricsHistory
from .recall_sparsity import recall_sparsity_curve
from .train import (
    TrainingState,
    close_training_state,
    create_training_state,
    default_batch_step,
    move_batch,
    resolve_device,
    resume_training_state,
    save_training_state,
    seed_everything,
    train_model,
)

__all__ = [name for name in dir() if not name.startswith("_")]
