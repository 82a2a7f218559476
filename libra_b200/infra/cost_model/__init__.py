"""Cost model, two-level optimizer and the Global Resource Planner."""

from libra_b200.infra.cost_model.global_resource_planner import (ElasticHybridSignal, GlobalResourcePlan,  # noqa: F401
                                                                  GlobalResourcePlanner, PlannerDecision,
                                                                  RuntimeResourceMetrics)
from libra_b200.infra.cost_model.model import (CostModel, RequestInfo, RolloutClusterConfig,  # noqa: F401
                                               TrainParallelConfig)
from libra_b200.infra.cost_model.optimizer import TwoLevelNestedOptimizer  # noqa: F401
