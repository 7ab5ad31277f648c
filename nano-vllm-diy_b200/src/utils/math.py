def divide(numerator: int, denominator: int) -> int:
    """Exact integer division, as src/utils/math.py:1-3 (asserts divisibility)."""
    assert numerator % denominator == 0, f"{numerator} is not divisible by {denominator}"
    return numerator // denominator
