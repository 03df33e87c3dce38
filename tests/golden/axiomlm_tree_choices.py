"""The reference's default Medusa tree (engine/medusa.py:28-45), as data."""

DEFAULT_MEDUSA_TREE_CHOICES = [
    (0,), (1,), (2,), (3,),
    (0, 0), (0, 1), (0, 2), (1, 0), (1, 1), (2, 0),
    (0, 0, 0), (0, 0, 1), (0, 1, 0), (0, 1, 1), (1, 0, 0),
    (0, 0, 0, 0),
]
