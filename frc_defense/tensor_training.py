"""`python -m frc_defense.tensor_training {train,evaluate,evaluate-game-ablations,curriculum}`."""
from autodrive_b200.train.cli import main, train  # noqa: F401
from autodrive_b200.train.evaluation import (  # noqa: F401
    evaluate, evaluate_game_ablations, evaluate_once as _evaluate_once, wilson_interval as _wilson_interval)
from autodrive_b200.train.generational import (  # noqa: F401
    dispatch_evaluations as _dispatch_opponent_evaluations, generational_train,
    select_checkpoint_population as _select_checkpoint_population)

if __name__ == "__main__":
    main()
