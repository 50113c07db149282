"""Command-line helpers of the reference that touch the candidate cache."""
