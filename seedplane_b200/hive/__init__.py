"""HIVE: the pull-based request pool, with one agent per GPU running the B200 engine."""
from .cost import CostEstimate, CostKey, MeasuredCostModel
from .pool import HiveAgent, HiveBroker, WorkFuture, WorkTile
from .scheduler import BatchPlan, plan_homogeneous_batch

__all__ = ["HiveAgent", "HiveBroker", "WorkFuture", "WorkTile", "CostEstimate", "CostKey", "MeasuredCostModel",
           "BatchPlan", "plan_homogeneous_batch"]
