"""Evaluation metrics."""

from .auc import StreamingHistogramAUC, TaskMonitor, binary_auc, group_auc, trapezoid_auc

__all__ = ["StreamingHistogramAUC", "TaskMonitor", "binary_auc", "group_auc", "trapezoid_auc"]
