"""Model-independent operators of the experimental layer."""
