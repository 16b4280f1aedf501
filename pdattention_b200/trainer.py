"""``PRAStandaloneTrainer``: object facade over the functional engine (``src/pra_torch/trainer.py``)."""

from __future__ import annotations

from pathlib import Path

from .config import CacheServiceConfig, PRAConfig, ResolverServiceConfig, TrainConfig
from .pra_train import create_pra_training_state, evaluate_pra_model, train_pra_model
from .runtime.train import resume_training_state, save_training_state


class PRAStandaloneTrainer:
    """Owns no algorithm: ``runtime.train`` optimises, ``pra_train`` builds caches and metrics."""

    def __init__(self, model_config: PRAConfig, train_config: TrainConfig, datamodule, *, model=None):
        self.model_config = model_config
        self.config = train_config
        self.datamodule = datamodule
        self.resolver_config = ResolverServiceConfig.from_value(train_config.resolver_config)
        self.cache_config = CacheServiceConfig.from_value(train_config.cache_config)
        self._state = create_pra_training_state(model_config, train_config, datamodule, model=model)
        self.trace_dir.mkdir(parents=True, exist_ok=True)

    model = property(lambda self: self._state.model)
    optimizer = property(lambda self: self._state.optimizer)
    scheduler = property(lambda self: self._state.scheduler)
    device = property(lambda self: self._state.device)
    run_dir = property(lambda self: self._state.run_dir)
    checkpoint = property(lambda self: self._state.checkpoint)
    global_step = property(lambda self: self._state.global_step)
    batch_step = property(lambda self: self._state.batch_step)
    start_epoch = property(lambda self: self._state.start_epoch)
    best_val_loss = property(lambda self: self._state.best_val_loss)

    @property
    def trace_dir(self) -> Path:
        return self.run_dir / "traces"

    def train(self) -> dict:
        result = train_pra_model(cfg=self.model_config, train_config=self.config, datamodule=self.datamodule,
                                 resolver_config=self.resolver_config, cache_config=self.cache_config,
                                 state=self._state)
        return {**result["test_metrics"], "timing_metrics": result["timing_metrics"]}

    def validate(self) -> dict:
        return self._evaluate(self.datamodule.val_loader(), "val")

    def test(self, save_predictions: str | None = None, save_traces: str | None = None) -> dict:
        return self._evaluate(self.datamodule.test_loader(), "test", save_predictions, save_traces)

    def resume(self, path) -> None:
        resume_training_state(self._state, path)

    def save(self, path, epoch: int) -> Path:
        return save_training_state(self._state, path, epoch)

    def _evaluate(self, loader, split, save_predictions=None, save_traces=None) -> dict:
        metrics = evaluate_pra_model(model=self.model, loader=loader, tokenizer=self.datamodule.tokenizer,
                                     train_config=self.config, device=self.device, split=split,
                                     resolver_config=self.resolver_config, cache_config=self.cache_config,
                                     save_predictions=save_predictions, save_traces=save_traces)
        if not self._state.logger_closed:
            self._state.logger.log_metrics(metrics, self.global_step, split)
        return metrics
