class CompilerParams:
    def __init__(self, **kwargs):
        self.kwargs = kwargs
