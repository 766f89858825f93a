from .activation import ReLU, Sigmoid, Softmax, Tanh
from .container import Sequential
from .linear import Flatten, Linear

__all__ = ["ReLU", "Sigmoid", "Softmax", "Tanh", "Sequential", "Flatten", "Linear"]
